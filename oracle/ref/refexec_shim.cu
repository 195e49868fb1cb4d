// refexec_shim.cu — C entry points over the reference's own GPU executor (src/native/executor.cpp:
// one k_conv3x3 / k_concat1x1 launch per plan step, buffers from src/native/layout.cpp), compiled
// for sm_100a from the reference sources by build.sh into oracle/_ref/libref_exec.so. With the
// reference's colour kernels (libref_kernels.so: aji_run_pre / aji_run_post) it is the reference's
// whole native video path on the B200 (src/aji_trt.cpp run_pre -> Executor::run -> run_post): the
// GPU bar bench.py times beside this engine. Benchmark and test infrastructure only.
#include <string>

#include "native/executor.h"
#include "refplan.h"

extern "C" void *ref_exec_create(const ref_step *steps, int nsteps, const int *channels, int nfeat, int depth_to_space,
                                 int unshuffle, int w, int h, void *stream, char *err, int err_size)
{
    std::string why;
    const ajinative::Plan p = ref_plan_of(steps, nsteps, channels, nfeat, depth_to_space, unshuffle);
    auto e = ajinative::Executor::create(p, w, h, (cudaStream_t)stream, &why);
    if (!e) {
        if (err && err_size > 0) {
            std::snprintf(err, (size_t)err_size, "%s", why.c_str());
        }
        return nullptr;
    }
    return e.release();
}

// in: NCHW fp16 [3][h][w]; out: NCHW fp16 [3][R h / u][R w / u]. Returns a cudaError_t.
extern "C" int ref_exec_run(void *e, const void *in, void *out, void *stream)
{
    return (int)static_cast<ajinative::Executor *>(e)->run(in, out, (cudaStream_t)stream);
}

extern "C" void ref_exec_release(void *e) { delete static_cast<ajinative::Executor *>(e); }
