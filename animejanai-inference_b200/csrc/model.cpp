/*
 * model.cpp — this engine's native model file and plan checks.
 *
 * File layout (little-endian):
 *   char magic[4] = "AJNM"; u32 version = 1;
 *   u32 nsteps, nfeat, unshuffle, depth_to_space; u32 name_len; char name[name_len];
 *   i32 channels[nfeat];
 *   per step:
 *     i32 kind (0 conv, 1 concat), in, act, gate, out, cin, cout, src, resid, dst, c, nsrc, srcs[4];
 *     i32 in_norm; f32 in_mean[3], in_scale[3]; i32 out_clamp;
 *     weights: i32 taps, cin, cout; u16 w[taps * cin * cout] ([taps][cin][cout], fp16 bits);
 *              f32 bias[cout]; i32 has_slope; f32 slope[cout] if has_slope;
 *     if gate == 2 (tanh 1x1): a second weights block (the attention conv).
 * The fields are those of the reference's PlanStep (src/native/lower.h:50-66); the Python side
 * writes it (animejanai-inference_b200/ajib.py, write_model) from the same structures the
 * reference's lowering produces for SRVGG Compact, SuperUltraCompact and SPAN.
 */
#include "onnx.h"
#include "plan.h"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>

namespace ajib {
namespace {

struct Reader {
    const unsigned char *p, *end;
    bool ok = true;
    template <typename T>
    T get()
    {
        T v{};
        if (p + sizeof(T) > end) {
            ok = false;
            return v;
        }
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    template <typename T>
    bool arr(std::vector<T> &v, size_t n)
    {
        if (n > (size_t)(end - p) / sizeof(T)) return ok = false;
        v.resize(n);
        std::memcpy(v.data(), p, n * sizeof(T));
        p += n * sizeof(T);
        return true;
    }
};

bool read_weights(Reader &r, PlanWeights &w)
{
    w.taps = r.get<int32_t>();
    w.cin = r.get<int32_t>();
    w.cout = r.get<int32_t>();
    if (!r.ok || (w.taps != 9 && w.taps != 1) || w.cin < 1 || w.cout < 1 || w.cin > 1024 || w.cout > 1024) return false;
    if (!r.arr(w.w, (size_t)w.taps * w.cin * w.cout) || !r.arr(w.bias, (size_t)w.cout)) return false;
    const int has_slope = r.get<int32_t>();
    if (has_slope && !r.arr(w.slope, (size_t)w.cout)) return false;
    return r.ok;
}

bool fail(std::string *why, const std::string &m)
{
    if (why) *why = m;
    return false;
}

}  // namespace

bool parse_model(const void *data, size_t size, Plan *out, std::string *why)
{
    Reader r{static_cast<const unsigned char *>(data), static_cast<const unsigned char *>(data) + size};
    char magic[4];
    for (char &c : magic) c = r.get<char>();
    if (!r.ok || std::memcmp(magic, "AJNM", 4) != 0) return fail(why, "not a native model file (magic)");
    if (r.get<uint32_t>() != 1) return fail(why, "unsupported native model file version");
    Plan p;
    const uint32_t nsteps = r.get<uint32_t>(), nfeat = r.get<uint32_t>();
    p.unshuffle = (int)r.get<uint32_t>();
    p.depth_to_space = (int)r.get<uint32_t>();
    const uint32_t name_len = r.get<uint32_t>();
    if (!r.ok || nsteps == 0 || nsteps > 4096 || nfeat > 4096 || name_len > 4096) return fail(why, "bad model header");
    std::vector<char> name;
    if (!r.arr(name, name_len)) return fail(why, "truncated model file");
    p.name.assign(name.begin(), name.end());
    std::vector<int32_t> ch;
    if (!r.arr(ch, nfeat)) return fail(why, "truncated model file");
    p.channels.assign(ch.begin(), ch.end());
    for (uint32_t i = 0; i < nsteps; i++) {
        PlanStep s;
        s.kind = (PlanStep::Kind)r.get<int32_t>();
        s.in = r.get<int32_t>();
        s.act = r.get<int32_t>();
        s.gate = r.get<int32_t>();
        s.out = r.get<int32_t>();
        s.cin = r.get<int32_t>();
        s.cout = r.get<int32_t>();
        s.src = r.get<int32_t>();
        s.resid = r.get<int32_t>();
        s.dst = r.get<int32_t>();
        s.c = r.get<int32_t>();
        s.nsrc = r.get<int32_t>();
        for (int &x : s.srcs) x = r.get<int32_t>();
        s.in_norm = r.get<int32_t>() != 0;
        for (float &x : s.in_mean) x = r.get<float>();
        for (float &x : s.in_scale) x = r.get<float>();
        s.out_clamp = r.get<int32_t>() != 0;
        if (!r.ok || !read_weights(r, s.w)) return fail(why, "truncated or bad step " + std::to_string(i));
        if (s.kind == PlanStep::CONV && s.gate == 2 && !read_weights(r, s.att))
            return fail(why, "truncated attention weights in step " + std::to_string(i));
        p.steps.push_back(std::move(s));
    }
    if (r.p != r.end) return fail(why, "trailing bytes after the last step");
    if (!validate_plan(p, why)) return false;
    *out = std::move(p);
    return true;
}

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

std::vector<uint8_t> serialize_model(const Plan &p)
{
    std::vector<uint8_t> b = {'A', 'J', 'N', 'M'};
    put<uint32_t>(b, 1);
    put<uint32_t>(b, (uint32_t)p.steps.size());
    put<uint32_t>(b, (uint32_t)p.channels.size());
    put<uint32_t>(b, (uint32_t)p.unshuffle);
    put<uint32_t>(b, (uint32_t)p.depth_to_space);
    put<uint32_t>(b, (uint32_t)p.name.size());
    b.insert(b.end(), p.name.begin(), p.name.end());
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
    return b;
}

bool load_model_bytes(const void *data, size_t size, Plan *out, std::string *why)
{
    if (size >= 4 && std::memcmp(data, "AJNM", 4) == 0) return parse_model(data, size, out, why);
    // otherwise an ONNX model: decoded and lowered to a plan
    OnnxModel m;
    std::string w;
    if (!parse_onnx(data, size, &m, &w)) return fail(why, "neither a native model file (magic AJNM) nor ONNX (" + w + ")");
    return lower_onnx(m, out, why);
}

bool load_model_file(const std::string &path, Plan *out, std::string *why)
{
    std::ifstream f(path, std::ios::binary);
    if (!f) return fail(why, "cannot read the model file " + path);
    std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    if (!load_model_bytes(bytes.data(), bytes.size(), out, why)) {
        if (why) *why = path + ": " + *why;
        return false;
    }
    return true;
}

// Structural checks: tensor ids in range and written before read, the model output written once
// by the last step, weight shapes matching the step.
bool validate_plan(const Plan &p, std::string *why)
{
    const int nf = (int)p.channels.size();
    std::vector<bool> written(nf, false);
    auto readable = [&](int t) { return t == kModelInput || (t >= 0 && t < nf && written[t]); };
    if (p.depth_to_space < 1 || p.depth_to_space > 4 || (p.unshuffle != 1 && p.unshuffle != 2) ||
        p.depth_to_space % p.unshuffle)
        return fail(why, "unsupported scale (depth-to-space 1..4, pixel-unshuffle 1 or 2, a whole scale)");
    for (size_t i = 0; i < p.steps.size(); i++) {
        const PlanStep &s = p.steps[i];
        const std::string at = "step " + std::to_string(i) + ": ";
        const bool last = i + 1 == p.steps.size();
        if (s.kind == PlanStep::CONCAT) {
            if (s.nsrc < 2 || s.nsrc > 4 || s.c < 8) return fail(why, at + "bad concat");
            for (int k = 0; k < s.nsrc; k++)
                if (!readable(s.srcs[k]) || s.srcs[k] < 0 || p.channels[s.srcs[k]] != s.c) return fail(why, at + "bad concat source");
            if (s.w.taps != 1 || s.w.cin != s.nsrc * s.c || s.w.cout != s.c) return fail(why, at + "concat weights do not match");
        } else if (s.kind == PlanStep::CONV) {
            if (s.w.taps != 9 || s.w.cin != s.cin || s.w.cout != s.cout) return fail(why, at + "conv weights do not match");
            if (s.in == 1 || s.in == 2) {
                if (s.src != kModelInput || s.cin != (s.in == 1 ? 3 : 12)) return fail(why, at + "bad conv source");
                if (p.unshuffle != s.in) return fail(why, at + "the model input's unshuffle does not match the plan's");
            } else if (s.in != 0 || !readable(s.src) || s.src < 0 || p.channels[s.src] != s.cin) {
                return fail(why, at + "bad conv source");
            }
            if (s.gate != 0 && (!readable(s.resid) || s.resid < 0 || p.channels[s.resid] != s.cout))
                return fail(why, at + "bad gate input");
            if (s.out != 0 && s.resid != -1 && s.resid != kModelInput) return fail(why, at + "bad skip input");
            if (s.out != 0 && s.resid == kModelInput && p.unshuffle != 1)
                return fail(why, at + "a model-input skip with a pixel-unshuffled input");
            if (s.gate == 2 && (s.att.taps != 1 || s.att.cin != s.cout || s.att.cout != s.cout))
                return fail(why, at + "the tanh gate's 1x1 weights do not match");
            if (s.act == 2 && s.w.slope.size() != (size_t)s.cout) return fail(why, at + "PReLU without slopes");
        } else {
            return fail(why, at + "unknown step kind");
        }
        if (last) {
            if (s.kind != PlanStep::CONV || s.out == 0 || s.dst != kModelOutput) return fail(why, "the last step must write the model output");
        } else {
            if (s.dst < 0 || s.dst >= nf || (s.kind == PlanStep::CONV && s.out != 0)) return fail(why, at + "bad destination");
            if (p.channels[s.dst] != (s.kind == PlanStep::CONCAT ? s.c : s.cout)) return fail(why, at + "destination width");
            written[s.dst] = true;
        }
    }
    const PlanStep &t = p.steps.back();
    const int r = t.out == 1 ? 2 : t.out == 2 ? 4 : t.out == 3 ? 1 : 3;
    if (r != p.depth_to_space) return fail(why, "depth-to-space factor does not match the output step");
    return true;
}

std::string describe(const Plan &p)
{
    int convs = 0, cats = 0, width = 0;
    for (const PlanStep &s : p.steps) {
        if (s.kind == PlanStep::CONCAT)
            cats++;
        else
            convs++;
        if (s.kind == PlanStep::CONV && s.out == 0) width = std::max(width, s.cout);
    }
    char b[256];
    std::snprintf(b, sizeof(b), "%s%s%d kernels (%d conv, %d concat), %d ch, %sdepth-to-space %d", p.name.c_str(),
                  p.name.empty() ? "" : ": ", convs + cats, convs, cats, width,
                  p.unshuffle > 1 ? "pixel-unshuffle 2, " : "", p.depth_to_space);
    return b;
}

double flops_per_pixel(const Plan &p)
{
    double f = 0;
    for (const PlanStep &s : p.steps) {
        f += 2.0 * s.w.taps * s.w.cin * s.w.cout;
        if (s.kind == PlanStep::CONV && s.gate == 2) f += 2.0 * s.att.cin * s.att.cout;
    }
    return f;
}

}  // namespace ajib
