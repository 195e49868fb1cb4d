/*
 * lower.cpp — an ONNX model (onnx.h) lowered to a native Plan (plan.h): the fused steps the
 * conv kernels run. The rules are those of the reference's lowering (src/native/lower.h, the
 * families its exporters produce); the code is this engine's own:
 *   - Conv 3x3 (stride 1, pad 1, one group) on the model input or a feature map is a conv step;
 *     what follows it folds into the step's epilogue:
 *       Relu -> ReLU; PRelu(slopes) / LeakyRelu(alpha) -> PReLU; Sigmoid(o) and Mul(o, s) -> SiLU;
 *       Add(x, o) with Sigmoid(o) -> Sub(., 0.5) -> Mul -> the SPAN gate (x a feature map);
 *       Add(x, o) with Conv1x1(o) -> Tanh -> Mul -> the SPANF3 gate;
 *       DepthToSpace by r (CRD; DCR by permuting the conv's output channels) -> the output step,
 *       optionally + Resize(model input) by nearest pixel replication (the SRVGG skip) and a
 *       final Clip(0, 1);
 *     a conv output the graph also needs unfolded (SPAN's last block c1, read by the concat
 *     before its activation) gets a second, plain step;
 *   - Conv1x1(Concat(f1..fn)), n = 2..4 -> a concat step;
 *   - the model input scaled and shifted by per-channel constants (Sub / Add / Mul / Div, e.g.
 *     SPAN's (x - mean) * 255) -> the normalisation the first conv applies where it loads;
 *   - the model input pixel-unshuffled by 2 (PyTorch's Reshape -> Transpose(0,1,3,5,2,4) ->
 *     Reshape, or SpaceToDepth 2 with its channels reordered) -> the first conv's unshuffled
 *     input (SPANF3: the conv runs at half resolution, 12 input channels);
 *   - Identity, Dropout and casts between float types pass through, and so do Pad and Slice
 *     whose amounts are computed from the input's shape or are zero / open-ended (an exporter's
 *     alignment to the unshuffle factor, which the even sizes the engine requires make a no-op);
 *     nodes off the data path (shape plumbing) are ignored; anything else on the data path
 *     refuses the model, with why.
 */
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "onnx.h"
#include "plan.h"

namespace ajib {
namespace {

uint16_t to_half(float f)
{
    // IEEE binary32 -> binary16, round to nearest even (the reference packs weights the same way)
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // 65520 and above round to infinity
    uint32_t v, rem, half;
    if (ax < 0x38800000u) {
        // a subnormal half: |f| / 2^-24 = m * 2^(e - 126) for the 24-bit significand m
        if (ax <= 0x33000000u) return (uint16_t)sign;  // at most 2^-25: rounds to zero (even)
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const int shift = 126 - (int)(ax >> 23);
        v = m >> shift;
        rem = m & ((1u << shift) - 1u);
        half = 1u << (shift - 1);
    } else {
        v = (ax >> 13) - (112u << 10);
        rem = ax & 0x1fffu;
        half = 0x1000u;
    }
    if (rem > half || (rem == half && (v & 1u))) v++;
    return (uint16_t)(sign | v);
}

bool float_cast(const OnnxNode &n)
{
    const int64_t to = n.attr_i("to", 0);
    return n.op == "Cast" && (to == kOnnxFloat || to == kOnnxFloat16 || to == kOnnxDouble || to == kOnnxBfloat16);
}

// ops whose data input is input 0 only (the rest are shapes, pads, scales, axes)
bool data_input0_only(const std::string &op)
{
    static const std::set<std::string> s = {"Reshape", "Pad", "Slice", "Transpose", "Cast", "Identity", "Dropout",
                                            "DepthToSpace", "SpaceToDepth", "Resize", "Expand", "Squeeze",
                                            "Unsqueeze", "Tile", "Upsample", "Clip"};
    return s.count(op) != 0;
}

// A nearest Resize by integer factor r that is pixel replication (output x reads input x / r).
// ONNX maps output x = r i + j to input i + (j + 0.5) / r - 0.5 (half_pixel, pytorch_half_pixel),
// which rounding to nearest takes to i, or to i + j / r (asymmetric), which floor takes to i (and
// round_prefer_floor only for r <= 2).
bool nearest_replicates(const OnnxNode &rz, int r)
{
    if (rz.op != "Resize" || rz.attr_s("mode", "nearest") != "nearest" || r < 1) return false;
    const std::string ct = rz.attr_s("coordinate_transformation_mode", "half_pixel");
    const std::string nm = rz.attr_s("nearest_mode", "round_prefer_floor");
    if (ct == "half_pixel" || ct == "pytorch_half_pixel") return nm == "round_prefer_floor" || nm == "round_prefer_ceil";
    if (ct == "asymmetric") return nm == "floor" || (nm == "round_prefer_floor" && r <= 2);
    return false;
}

struct Lowering {
    const OnnxModel &m;
    Plan &plan;
    std::string why;
    std::map<std::string, int> producer;               // tensor -> node
    std::map<std::string, std::string> alias;          // pass-through output -> its input
    std::map<std::string, std::vector<int>> consumers; // canonical tensor -> data nodes reading it
    std::set<std::string> data;                        // canonical data-path tensors
    std::vector<bool> done;
    std::string X, Y;                                  // canonical model input / output
    std::map<std::string, int> feat;                   // canonical tensor -> feature id
    bool norm = false;
    float mean[3] = {0.f, 0.f, 0.f}, scale[3] = {1.f, 1.f, 1.f};
    std::string Xn;                                    // canonical normalised model input
    struct Unshuffled {
        bool dcr = false;     // SpaceToDepth order: channel (ry * 2 + rx) * 3 + c
        bool normed = false;  // of the normalised model input
    };
    std::map<std::string, Unshuffled> unshuffled;      // canonical tensor -> the unshuffled input

    Lowering(const OnnxModel &m_, Plan &p) : m(m_), plan(p), done(m_.nodes.size(), false) {}

    bool fail(const std::string &msg)
    {
        if (why.empty()) why = msg;
        return false;
    }
    std::string canon(std::string t) const
    {
        for (auto it = alias.find(t); it != alias.end(); it = alias.find(t)) t = it->second;
        return t;
    }
    const OnnxNode &node(int i) const { return m.nodes[(size_t)i]; }
    std::vector<int> uses(const std::string &t) const
    {
        const auto it = consumers.find(canon(t));
        return it == consumers.end() ? std::vector<int>() : it->second;
    }
    // the input of binary node n other than t, or ""
    std::string other(int n, const std::string &t) const
    {
        const OnnxNode &b = node(n);
        if (b.in.size() != 2) return "";
        const std::string a = canon(b.in[0]), c = canon(b.in[1]), tt = canon(t);
        return a == tt ? c : c == tt ? a : "";
    }
    const OnnxTensor *constant(const std::string &name) const
    {
        const auto it = m.inits.find(name);
        if (it != m.inits.end()) return &it->second;
        const auto p = producer.find(name);
        if (p == producer.end()) return nullptr;
        const OnnxNode &n = node(p->second);
        if (n.op == "Constant") {
            const OnnxAttr *v = n.attr("value");
            return v && v->type == 4 ? &v->t : nullptr;
        }
        // an exporter's Unsqueeze / Reshape / Cast of an initializer (a PReLU slope): the same values
        if ((n.op == "Unsqueeze" || n.op == "Reshape" || n.op == "Squeeze" || float_cast(n)) && !n.in.empty())
            return constant(n.in[0]);
        return nullptr;
    }
    bool floats(const std::string &name, std::vector<float> *v) const
    {
        const auto p = producer.find(name);
        if (p != producer.end() && node(p->second).op == "Constant") {
            const OnnxAttr *f = node(p->second).attr("value_float");
            if (f) {
                *v = {f->f};
                return true;
            }
        }
        const OnnxTensor *t = constant(name);
        return t && t->to_floats(v);
    }

    bool ints(const std::string &name, std::vector<int64_t> *v) const
    {
        const OnnxTensor *t = constant(name);
        return t && t->to_ints(v);
    }

    // Pad / Slice on the data path pass through when they only align the input to the unshuffle
    // factor: amounts computed at run time (from Shape), zero pads, slices from 0 to an open end
    // (reference src/native/lower.cpp pass_through_ok).
    bool pass_through_ok(const OnnxNode &n)
    {
        if (n.op == "Pad") {
            if (n.in.size() < 2 || n.in[1].empty()) {
                for (int64_t p : n.attr_ints("pads"))
                    if (p != 0) return fail("Pad by a fixed amount");
                return true;
            }
            std::vector<int64_t> v;
            if (!constant(n.in[1])) return true;  // computed from the input's shape
            if (!ints(n.in[1], &v)) return fail("Pad by a fixed amount");
            for (int64_t p : v)
                if (p != 0) return fail("Pad by a fixed amount");
            return true;
        }
        // Slice
        if (n.in.size() < 3) return fail("Slice without starts/ends");
        std::vector<int64_t> st, en, sp;
        if (constant(n.in[1])) {
            if (!ints(n.in[1], &st)) return fail("Slice that crops the start");
            for (int64_t x : st)
                if (x != 0) return fail("Slice that crops the start");
        }
        if (n.in.size() > 4 && !n.in[4].empty()) {
            if (!ints(n.in[4], &sp)) return fail("strided Slice");
            for (int64_t x : sp)
                if (x != 1) return fail("strided Slice");
        }
        if (constant(n.in[2])) {
            if (!ints(n.in[2], &en)) return fail("Slice by a fixed size");
            for (int64_t x : en)
                if (x < (int64_t(1) << 30)) return fail("Slice by a fixed size");
        }
        return true;
    }

    // the sole data node reading t, if it is an op, else -1
    int sole(const std::string &t, const char *op) const
    {
        const std::vector<int> u = uses(t);
        return u.size() == 1 && node(u[0]).op == op ? u[0] : -1;
    }

    // Reshape -> Transpose(0,1,3,5,2,4) -> Reshape of the model input: PyTorch's pixel_unshuffle(2)
    bool lower_unshuffle_reshape(int ri)
    {
        const OnnxNode &r1 = node(ri);
        const int t = sole(r1.out[0], "Transpose");
        if (t < 0) return fail("a Reshape of the model input that is not a pixel-unshuffle");
        if (node(t).attr_ints("perm") != std::vector<int64_t>{0, 1, 3, 5, 2, 4})
            return fail("a Reshape / Transpose of the model input that is not a pixel-unshuffle");
        const int r2 = sole(node(t).out[0], "Reshape");
        if (r2 < 0) return fail("a Reshape / Transpose of the model input that is not a pixel-unshuffle");
        done[(size_t)ri] = done[(size_t)t] = done[(size_t)r2] = true;
        Unshuffled u;
        u.normed = !Xn.empty() && canon(r1.in[0]) == Xn;
        unshuffled[canon(node(r2).out[0])] = u;
        return true;
    }

    bool lower_space_to_depth(int si)
    {
        const OnnxNode &n = node(si);
        if (n.attr_i("blocksize", 0) != 2) return fail("SpaceToDepth other than 2x on the model input");
        done[(size_t)si] = true;
        Unshuffled u;
        u.dcr = true;
        u.normed = !Xn.empty() && canon(n.in[0]) == Xn;
        unshuffled[canon(n.out[0])] = u;
        return true;
    }

    int new_feature(const std::string &t, int c)
    {
        plan.channels.push_back(c);
        const int id = (int)plan.channels.size() - 1;
        feat[canon(t)] = id;
        return id;
    }

    bool conv_weights(const OnnxNode &cv, int k, PlanWeights *w, int *cin, int *cout)
    {
        if (cv.in.size() < 2) return fail("Conv without weights");
        const OnnxTensor *W = constant(cv.in[1]);
        std::vector<float> wf, bf;
        if (!W || W->dims.size() != 4 || !W->to_floats(&wf)) return fail("Conv weights are not a constant 4-D tensor");
        if (W->dims[2] != k || W->dims[3] != k) return fail("Conv kernel is not " + std::to_string(k) + "x" + std::to_string(k));
        if (cv.attr_i("group", 1) != 1) return fail("grouped Conv");
        for (int64_t s : cv.attr_ints("strides"))
            if (s != 1) return fail("strided Conv");
        for (int64_t d : cv.attr_ints("dilations"))
            if (d != 1) return fail("dilated Conv");
        const std::vector<int64_t> pads = cv.attr_ints("pads");
        const std::string ap = cv.attr_s("auto_pad", "NOTSET");
        const int want = k / 2;
        if (ap == "SAME_UPPER" || ap == "SAME_LOWER") {
        } else if (ap != "NOTSET" && ap != "") {
            return fail("Conv auto_pad " + ap);
        } else {
            if (pads.empty() ? want != 0 : pads.size() != 4) return fail("Conv padding");
            for (int64_t p : pads)
                if (p != want) return fail("Conv padding is not " + std::to_string(want));
        }
        *cout = (int)W->dims[0];
        *cin = (int)W->dims[1];
        w->taps = k * k;
        w->cin = *cin;
        w->cout = *cout;
        w->w.assign((size_t)k * k * *cin * *cout, 0);
        for (int o = 0; o < *cout; o++)
            for (int i = 0; i < *cin; i++)
                for (int t = 0; t < k * k; t++)
                    w->w[((size_t)t * *cin + i) * *cout + o] = to_half(wf[((size_t)o * *cin + i) * k * k + t]);
        w->bias.assign(*cout, 0.f);
        if (cv.in.size() > 2 && !cv.in[2].empty()) {
            if (!floats(cv.in[2], &bf) || (int)bf.size() != *cout) return fail("Conv bias");
            w->bias = bf;
        }
        return true;
    }

    // Lower Conv node ci (3x3) and what folds into it.
    bool lower_conv(int ci)
    {
        const OnnxNode &cv = node(ci);
        done[(size_t)ci] = true;
        PlanStep st;
        st.kind = PlanStep::CONV;
        if (!conv_weights(cv, 3, &st.w, &st.cin, &st.cout)) return false;
        const std::string src = canon(cv.in[0]);
        if (src == X || src == Xn) {
            if (st.cin != 3) return fail("the first conv reads " + std::to_string(st.cin) + " input channels, not RGB");
            st.in = AJIB_IN_NCHW3;
            st.src = kModelInput;
            if (src == Xn && norm) {
                st.in_norm = true;
                for (int c = 0; c < 3; c++) {
                    st.in_mean[c] = mean[c];
                    st.in_scale[c] = scale[c];
                }
            }
        } else if (unshuffled.count(src)) {
            const Unshuffled u = unshuffled[src];
            if (st.cin != 12) return fail("the first conv of an unshuffled input reads " + std::to_string(st.cin) + " channels, not 12");
            st.in = AJIB_IN_NCHW3_UNSHUFFLE2;
            st.src = kModelInput;
            plan.unshuffle = 2;
            if (u.dcr) {
                // SpaceToDepth's channel (ry * 2 + rx) * 3 + c is the kernel's c * 4 + ry * 2 + rx
                PlanWeights w2 = st.w;
                for (int k = 0; k < 12; k++) {
                    const int from = ((k % 4) / 2 * 2 + k % 2) * 3 + k / 4;
                    for (int t = 0; t < 9; t++)
                        for (int o = 0; o < st.cout; o++)
                            w2.w[((size_t)t * 12 + k) * st.cout + o] = st.w.w[((size_t)t * 12 + from) * st.cout + o];
                }
                st.w = w2;
            }
            if (u.normed && norm) {
                st.in_norm = true;
                for (int c = 0; c < 3; c++) {
                    st.in_mean[c] = mean[c];
                    st.in_scale[c] = scale[c];
                }
            }
        } else {
            const auto f = feat.find(src);
            if (f == feat.end()) return fail("a Conv reads a tensor that is not a feature map");
            st.in = AJIB_IN_NHWC;
            st.src = f->second;
        }
        std::string o = canon(cv.out[0]);
        std::vector<int> us = uses(o);
        auto take = [&](int n) { done[(size_t)n] = true; };
        auto op_of = [&](int n) -> const std::string & { return node(n).op; };

        // the output step: DepthToSpace [+ Resize skip] [+ Clip], or the 3-channel output itself
        if (us.size() == 1 && op_of(us[0]) == "DepthToSpace") {
            const OnnxNode &d2s = node(us[0]);
            const int r = (int)d2s.attr_i("blocksize", 0);
            if (r < 1 || r > 4 || st.cout != 3 * r * r) return fail("DepthToSpace by " + std::to_string(r));
            if (d2s.attr_s("mode", "DCR") == "DCR" && r > 1) {
                // DCR reads channel (ry * r + rx) * 3 + c: reorder to CRD's c * r * r + ry * r + rx
                PlanWeights w2 = st.w;
                for (int c = 0; c < 3; c++)
                    for (int q = 0; q < r * r; q++) {
                        const int from = q * 3 + c, to = c * r * r + q;
                        for (size_t t = 0; t < (size_t)9 * st.cin; t++) w2.w[t * st.cout + to] = st.w.w[t * st.cout + from];
                        w2.bias[to] = st.w.bias[from];
                    }
                st.w = w2;
            }
            take(us[0]);
            st.out = r == 2 ? AJIB_OUT_D2S2 : r == 4 ? AJIB_OUT_D2S4 : r == 1 ? AJIB_OUT_D2S1 : AJIB_OUT_D2S3;
            plan.depth_to_space = r;
            return finish_output(st, canon(d2s.out[0]), r);
        }
        if (st.cout == 3 && (o == Y || (us.size() == 1 && op_of(us[0]) == "Clip"))) {
            st.out = AJIB_OUT_D2S1;
            plan.depth_to_space = 1;
            return finish_output(st, o, 1);
        }

        // activations and gates
        std::string result = o;
        bool raw_needed = false;  // o itself is read by a node outside the folded pattern
        std::vector<int> folded;
        if (us.size() == 1 && op_of(us[0]) == "Relu") {
            st.act = AJIB_ACT_RELU;
            folded = {us[0]};
            result = canon(node(us[0]).out[0]);
        } else if (us.size() == 1 && (op_of(us[0]) == "PRelu" || op_of(us[0]) == "LeakyRelu")) {
            const OnnxNode &a = node(us[0]);
            std::vector<float> sl;
            if (a.op == "PRelu") {
                if (a.in.size() != 2 || !floats(a.in[1], &sl)) return fail("PRelu slopes are not constant");
            } else {
                const OnnxAttr *al = a.attr("alpha");
                sl = {al ? al->f : 0.01f};
            }
            if (sl.size() == 1) sl.assign(st.cout, sl[0]);
            if ((int)sl.size() != st.cout) return fail("PRelu slopes do not match the channels");
            st.act = AJIB_ACT_PRELU;
            st.w.slope = sl;
            folded = {us[0]};
            result = canon(node(us[0]).out[0]);
        } else {
            // SiLU: Sigmoid(o) and Mul(o, Sigmoid(o)); SPAN gate: Add(x, o), Sigmoid(o) -> Sub 0.5 -> Mul;
            // SPANF3 gate: Add(x, o), Conv1x1(o) -> Tanh -> Mul
            int sig = -1, add = -1, att = -1;
            std::vector<int> rest;
            for (int n : us) {
                if (op_of(n) == "Sigmoid" && sig < 0) sig = n;
                else if (op_of(n) == "Add" && add < 0) add = n;
                else if (op_of(n) == "Conv" && att < 0 && !node(n).in.empty() && canon(node(n).in[0]) == o) att = n;
                else rest.push_back(n);
            }
            int silu_mul = -1;
            if (sig >= 0) {
                for (int n : rest)
                    if (op_of(n) == "Mul" && other(n, o) == canon(node(sig).out[0])) silu_mul = n;
            }
            if (sig >= 0 && silu_mul >= 0 && add < 0 && att < 0) {
                st.act = AJIB_ACT_SILU;
                folded = {sig, silu_mul};
                rest.erase(std::remove(rest.begin(), rest.end(), silu_mul), rest.end());
                raw_needed = !rest.empty();
                result = canon(node(silu_mul).out[0]);
            } else if (add >= 0 && (sig >= 0 || att >= 0) && rest.empty()) {
                const std::string x = other(add, o);
                const auto fx = feat.find(x);
                if (fx == feat.end()) return fail("a gate's block input is not a feature map");
                const std::string sum = canon(node(add).out[0]);
                int mul = -1;
                std::vector<int> gate_nodes = {add};
                if (sig >= 0) {
                    const std::vector<int> su = uses(node(sig).out[0]);
                    if (su.size() != 1 || op_of(su[0]) != "Sub") return fail("sigmoid gate without Sub 0.5");
                    std::vector<float> half;
                    const OnnxNode &sub = node(su[0]);
                    if (sub.in.size() != 2 || canon(sub.in[0]) != canon(node(sig).out[0]) || !floats(sub.in[1], &half) ||
                        half.size() != 1 || half[0] != 0.5f)
                        return fail("sigmoid gate without Sub 0.5");
                    const std::vector<int> mu = uses(sub.out[0]);
                    if (mu.size() != 1 || op_of(mu[0]) != "Mul" || other(mu[0], sub.out[0]) != sum)
                        return fail("sigmoid gate without its Mul");
                    mul = mu[0];
                    gate_nodes.insert(gate_nodes.end(), {sig, su[0], mul});
                    st.gate = AJIB_GATE_SIGMOID_HALF;
                } else {
                    int acin = 0, acout = 0;
                    if (!conv_weights(node(att), 1, &st.att, &acin, &acout) || acin != st.cout || acout != st.cout)
                        return fail("SPANF3 gate's 1x1 conv");
                    const std::vector<int> tu = uses(node(att).out[0]);
                    if (tu.size() != 1 || op_of(tu[0]) != "Tanh") return fail("SPANF3 gate without Tanh");
                    const std::vector<int> mu = uses(node(tu[0]).out[0]);
                    if (mu.size() != 1 || op_of(mu[0]) != "Mul" || other(mu[0], node(tu[0]).out[0]) != sum)
                        return fail("SPANF3 gate without its Mul");
                    mul = mu[0];
                    gate_nodes.insert(gate_nodes.end(), {att, tu[0], mul});
                    st.gate = AJIB_GATE_TANH1X1;
                }
                if (uses(sum).size() != 1) return fail("a gate's sum is read elsewhere");
                st.resid = fx->second;
                folded = gate_nodes;
                result = canon(node(mul).out[0]);
            } else if (us.size() == 1 && op_of(us[0]) == "Add" && feat.count(other(us[0], o))) {
                st.gate = AJIB_GATE_RESIDUAL;
                st.resid = feat[other(us[0], o)];
                folded = {us[0]};
                result = canon(node(us[0]).out[0]);
            }
        }
        for (int n : folded) take(n);
        if (result == o && st.act == 0 && st.gate == 0) raw_needed = false;
        if (raw_needed) {
            // a plain copy of the step for the unfolded value
            PlanStep rawst = st;
            rawst.act = AJIB_ACT_NONE;
            rawst.w.slope.clear();
            rawst.dst = new_feature(o, st.cout);
            plan.steps.push_back(rawst);
        }
        st.dst = new_feature(result, st.cout);
        plan.steps.push_back(st);
        return true;
    }

    // The output step: its skip (Add with the nearest-upsampled model input) and clamp, up to
    // the graph output.
    bool finish_output(PlanStep st, std::string t, int r)
    {
        std::vector<int> us = uses(t);
        if (us.size() == 1 && node(us[0]).op == "Add") {
            const int add = us[0];
            const std::string s = other(add, t);
            const auto p = producer.find(s);
            // the skip: Resize(model input) by r, or the model input itself at r == 1
            bool skip = false;
            if (r == 1 && (s == X)) skip = true;
            if (!skip && p != producer.end() && nearest_replicates(node(p->second), r) && !node(p->second).in.empty() &&
                canon(node(p->second).in[0]) == X) {
                skip = true;
                done[(size_t)p->second] = true;
            }
            if (!skip) return fail("the output adds something other than the upsampled model input");
            done[(size_t)add] = true;
            st.resid = kModelInput;
            t = canon(node(add).out[0]);
            us = uses(t);
        }
        if (us.size() == 1 && node(us[0]).op == "Clip") {
            const OnnxNode &cl = node(us[0]);
            std::vector<float> lo, hi;
            float a = cl.attr("min") ? cl.attr("min")->f : -INFINITY, b = cl.attr("max") ? cl.attr("max")->f : INFINITY;
            if (cl.in.size() > 1 && !cl.in[1].empty() && floats(cl.in[1], &lo) && lo.size() == 1) a = lo[0];
            if (cl.in.size() > 2 && !cl.in[2].empty() && floats(cl.in[2], &hi) && hi.size() == 1) b = hi[0];
            if (a != 0.f || b != 1.f) return fail("the output is clipped to other than [0, 1]");
            done[(size_t)us[0]] = true;
            st.out_clamp = true;
            t = canon(cl.out[0]);
            us = uses(t);
        }
        if (t != Y || !us.empty()) return fail("the output step does not produce the model output");
        st.dst = kModelOutput;
        plan.steps.push_back(st);
        return true;
    }

    bool lower_concat(int ci)
    {
        const OnnxNode &cat = node(ci);
        done[(size_t)ci] = true;
        if (cat.attr_i("axis", 1) != 1) return fail("Concat not over channels");
        const int n = (int)cat.in.size();
        if (n < 2 || n > 4) return fail("Concat of " + std::to_string(n) + " maps");
        const std::vector<int> us = uses(cat.out[0]);
        if (us.size() != 1 || node(us[0]).op != "Conv") return fail("a Concat not read by one 1x1 Conv");
        PlanStep st;
        st.kind = PlanStep::CONCAT;
        int cin = 0, cout = 0;
        if (!conv_weights(node(us[0]), 1, &st.w, &cin, &cout)) return false;
        st.nsrc = n;
        st.c = cout;
        st.cin = cin;
        st.cout = cout;
        for (int k = 0; k < n; k++) {
            const auto f = feat.find(canon(cat.in[(size_t)k]));
            if (f == feat.end()) return fail("a Concat input is not a feature map");
            if (plan.channels[(size_t)f->second] != cout) return fail("Concat inputs are not as wide as its output");
            st.srcs[k] = f->second;
        }
        if (cin != n * cout) return fail("the Concat's 1x1 conv does not read all inputs");
        done[(size_t)us[0]] = true;
        st.dst = new_feature(node(us[0]).out[0], cout);
        plan.steps.push_back(st);
        return true;
    }

    // Sub / Add / Mul / Div of the model input by per-channel constants
    bool lower_norm(int ni)
    {
        const OnnxNode &n = node(ni);
        const std::string in = canon(n.in[0]) == (Xn.empty() ? X : Xn) ? n.in[1] : n.in[0];
        std::vector<float> c;
        if (!floats(in, &c) || (c.size() != 1 && c.size() != 3)) return fail(n.op + " of the model input by a non-constant");
        if (c.size() == 1) c.assign(3, c[0]);
        if (canon(n.in[1]) == (Xn.empty() ? X : Xn) && (n.op == "Sub" || n.op == "Div"))
            return fail(n.op + " with the model input second");
        for (int k = 0; k < 3; k++) {
            // value = (x - mean) * scale
            if (n.op == "Sub") mean[k] += c[k] / scale[k];
            else if (n.op == "Add") mean[k] -= c[k] / scale[k];
            else if (n.op == "Mul") scale[k] *= c[k];
            else scale[k] /= c[k];
            if (!(scale[k] != 0.f) || !std::isfinite(scale[k]) || !std::isfinite(mean[k])) return fail("input normalisation");
        }
        norm = true;
        done[(size_t)ni] = true;
        Xn = canon(n.out[0]);
        return true;
    }

    bool run()
    {
        if (m.inputs.size() != 1 || m.outputs.size() != 1) return fail("the model must have one input and one output");
        for (size_t i = 0; i < m.nodes.size(); i++)
            for (const std::string &o : m.nodes[i].out) producer[o] = (int)i;
        // pass-through ops alias their output to their input
        for (const OnnxNode &n : m.nodes)
            if ((n.op == "Identity" || n.op == "Dropout" || float_cast(n) || n.op == "Pad" || n.op == "Slice") &&
                !n.in.empty() && !n.out.empty())
                alias[n.out[0]] = n.in[0];
        X = canon(m.inputs[0]);
        Y = canon(m.outputs[0]);
        // the data path: tensors computed from the model input
        data.insert(X);
        for (size_t i = 0; i < m.nodes.size(); i++) {
            const OnnxNode &n = m.nodes[i];
            // shape values are not data, whatever they were computed from
            if (n.op == "Shape" || n.op == "Size") continue;
            bool reads = false;
            for (size_t k = 0; k < n.in.size(); k++) {
                if (k > 0 && data_input0_only(n.op)) break;
                if (!n.in[k].empty() && data.count(canon(n.in[k]))) reads = true;
            }
            if (!reads) continue;
            // a pass-through node is its input under another name: not a consumer
            const bool through = n.op == "Identity" || n.op == "Dropout" || float_cast(n) || n.op == "Pad" || n.op == "Slice";
            for (size_t k = 0; k < n.in.size() && !through; k++)
                if (!n.in[k].empty() && data.count(canon(n.in[k])) && !(k > 0 && data_input0_only(n.op)))
                    consumers[canon(n.in[k])].push_back((int)i);
            for (const std::string &o : n.out) data.insert(canon(o));
        }
        for (size_t i = 0; i < m.nodes.size(); i++) {
            const OnnxNode &n = m.nodes[i];
            if (done[i] || n.out.empty() || !data.count(canon(n.out[0]))) continue;
            if (n.op == "Identity" || n.op == "Dropout" || float_cast(n)) continue;
            if (n.op == "Pad" || n.op == "Slice") {
                if (!pass_through_ok(n)) return false;
                continue;
            }
            bool ok;
            const std::string in0 = n.in.empty() ? "" : canon(n.in[0]), in1 = n.in.size() > 1 ? canon(n.in[1]) : "";
            const std::string cur_in = Xn.empty() ? X : Xn;
            if (n.op == "Conv") {
                ok = lower_conv((int)i);
            } else if (n.op == "Concat") {
                ok = lower_concat((int)i);
            } else if ((n.op == "Sub" || n.op == "Add" || n.op == "Mul" || n.op == "Div") &&
                       (in0 == cur_in || in1 == cur_in) && plan.steps.empty()) {
                ok = lower_norm((int)i);
            } else if (n.op == "Resize" && in0 == X) {
                continue;  // the skip, taken by the output step
            } else if (n.op == "Reshape" && in0 == cur_in && plan.steps.empty()) {
                ok = lower_unshuffle_reshape((int)i);
            } else if (n.op == "SpaceToDepth" && in0 == cur_in && plan.steps.empty()) {
                ok = lower_space_to_depth((int)i);
            } else {
                return fail("op " + n.op + " on the data path is not supported by the native kernels");
            }
            if (!ok) return false;
        }
        if (plan.steps.empty() || plan.steps.back().dst != kModelOutput) return fail("no output step");
        for (size_t i = 0; i < m.nodes.size(); i++) {
            const OnnxNode &n = m.nodes[i];
            if (!done[i] && !n.out.empty() && data.count(canon(n.out[0])) && n.op == "Resize" && !n.in.empty() &&
                canon(n.in[0]) == X)
                return fail("a Resize of the model input that is not the output's skip");
        }
        return true;
    }
};

}  // namespace

bool lower_onnx(const OnnxModel &m, Plan *plan, std::string *why)
{
    *plan = Plan();
    plan->name = "onnx";
    Lowering L(m, *plan);
    if (!L.run()) {
        if (why) *why = "ONNX model not lowered: " + L.why;
        return false;
    }
    std::string v;
    if (!validate_plan(*plan, &v)) {
        if (why) *why = "ONNX model lowered to an invalid plan: " + v;
        return false;
    }
    return true;
}

}  // namespace ajib
