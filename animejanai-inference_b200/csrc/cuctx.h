/*
 * cuctx.h — the few CUDA driver calls the front-ends need (context retain / push / pop), resolved
 * at run time through the runtime's driver entry-point query so the library has no link-time
 * dependency on libcuda (it still loads on a machine without a GPU, where only symbol checks run).
 */
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace ajib {

struct Driver {
    CUresult (*init)(unsigned) = nullptr;
    CUresult (*device_get)(CUdevice *, int) = nullptr;
    CUresult (*primary_retain)(CUcontext *, CUdevice) = nullptr;
    CUresult (*primary_release)(CUdevice) = nullptr;
    CUresult (*push)(CUcontext) = nullptr;
    CUresult (*pop)(CUcontext *) = nullptr;
    CUresult (*ctx_get_device)(CUdevice *) = nullptr;
    CUresult (*ctx_get_current)(CUcontext *) = nullptr;
    bool ok = false;
};

inline const Driver &driver()
{
    static const Driver d = [] {
        Driver r;
        auto get = [](const char *name, void **fn) {
            cudaDriverEntryPointQueryResult q;
            return cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess;
        };
        r.ok = get("cuInit", (void **)&r.init) && get("cuDeviceGet", (void **)&r.device_get) &&
               get("cuDevicePrimaryCtxRetain", (void **)&r.primary_retain) &&
               get("cuDevicePrimaryCtxRelease", (void **)&r.primary_release) &&
               get("cuCtxPushCurrent", (void **)&r.push) && get("cuCtxPopCurrent", (void **)&r.pop) &&
               get("cuCtxGetDevice", (void **)&r.ctx_get_device) && get("cuCtxGetCurrent", (void **)&r.ctx_get_current);
        return r;
    }();
    return d;
}

// Makes ctx current for the guard's scope (like the reference's CtxGuard, src/aji_trt.cpp).
class CtxGuard {
public:
    explicit CtxGuard(CUcontext c)
    {
        const Driver &d = driver();
        ok = d.ok && c && d.push(c) == CUDA_SUCCESS;
    }
    ~CtxGuard()
    {
        if (ok) {
            CUcontext prev;
            driver().pop(&prev);
        }
    }
    bool ok = false;
};

}  // namespace ajib
