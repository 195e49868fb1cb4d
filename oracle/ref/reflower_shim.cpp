// reflower_shim.cpp — C entry point over the reference's ONNX lowering (src/native/onnx_graph.cpp
// parse_onnx + src/native/lower.cpp lower, with the CUDA kernel widths), compiled from the
// reference sources by build.sh into oracle/_ref/libref_lower.so: the checker of this engine's
// lowering. It writes the reference's Plan in this engine's native model file layout (the fields
// are the same PlanStep fields), so the two lowerings compare byte for byte. Test infrastructure
// only.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "native/lower.h"
#include "native/onnx_graph.h"

using namespace ajinative;

namespace {

template <typename T>
void put(std::vector<uint8_t> &b, const T &v)
{
    const uint8_t *p = reinterpret_cast<const uint8_t *>(&v);
    b.insert(b.end(), p, p + sizeof(T));
}

template <typename T>
void put_all(std::vector<uint8_t> &b, const std::vector<T> &v)
{
    const uint8_t *p = reinterpret_cast<const uint8_t *>(v.data());
    b.insert(b.end(), p, p + v.size() * sizeof(T));
}

void put_weights(std::vector<uint8_t> &b, const PlanWeights &w)
{
    put<int32_t>(b, w.taps);
    put<int32_t>(b, w.cin);
    put<int32_t>(b, w.cout);
    put_all(b, w.w);
    put_all(b, w.bias);
    put<int32_t>(b, w.slope.empty() ? 0 : 1);
    put_all(b, w.slope);
}

}  // namespace

extern "C" int ref_lower(const void *data, size_t n, void *out, size_t cap, size_t *size, char *why, size_t why_cap)
{
    OnnxGraph g;
    Plan p;
    std::string w;
    if (!parse_onnx(data, n, &g, &w) || !lower(g, &p, &w, kernel_widths_cuda())) {
        if (why && why_cap) std::snprintf(why, why_cap, "%s", w.c_str());
        return -1;
    }
    std::vector<uint8_t> b = {'A', 'J', 'N', 'M'};
    put<uint32_t>(b, 1);
    put<uint32_t>(b, (uint32_t)p.steps.size());
    put<uint32_t>(b, (uint32_t)p.channels.size());
    put<uint32_t>(b, (uint32_t)p.unshuffle);
    put<uint32_t>(b, (uint32_t)p.depth_to_space);
    put<uint32_t>(b, 0);  // no name
    for (int c : p.channels) put<int32_t>(b, c);
    for (const PlanStep &s : p.steps) {
        for (int v : {(int)s.kind, s.in, s.act, s.gate, s.out, s.cin, s.cout, s.src, s.resid, s.dst, s.c, s.nsrc}) put<int32_t>(b, v);
        for (int x : s.srcs) put<int32_t>(b, x);
        put<int32_t>(b, s.in_norm ? 1 : 0);
        for (float x : s.in_mean) put<float>(b, x);
        for (float x : s.in_scale) put<float>(b, x);
        put<int32_t>(b, s.out_clamp ? 1 : 0);
        put_weights(b, s.w);
        if (s.kind == PlanStep::CONV && s.gate == 2) put_weights(b, s.att);
    }
    if (size) *size = b.size();
    if (out && cap >= b.size()) std::memcpy(out, b.data(), b.size());
    return 0;
}
