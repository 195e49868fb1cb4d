/*
 * executor.cpp — see plan.h. Reference: src/native/executor.cpp:23-127 (create/run) and
 * src/native/layout.cpp:10-77 (buffer assignment with lifetime reuse).
 */
#include "plan.h"

#include <algorithm>
#include <cstring>
#include <utility>

namespace ajib {

Executor::~Executor()
{
    for (cudaEvent_t e : prof_ev_)
        if (e) cudaEventDestroy(e);
    for (void *b : buffers_) cudaFree(b);
    for (Step &s : steps_) {
        ajib_weights_release(&s.w);
        ajib_weights_release(&s.att);
        cudaFree(s.pack_buf);
    }
}

const void *Executor::ptr(int t, const void *in, void *out) const
{
    if (t == kModelInput) return in;
    if (t == kModelOutput) return out;
    return t >= 0 ? tensor_[t] : nullptr;
}

int Executor::launches_per_run() const
{
    int n = 0;
    for (const Step &st : steps_) n += st.pack ? 2 : 1;  // the head's input pack is a launch of its own
    return n * bands_;
}

int Executor::launches_per_run_packed() const
{
    return launches_per_run() - (input_pack(nullptr) ? bands_ : 0);
}

std::unique_ptr<Executor> Executor::create(const Plan &plan, int in_w, int in_h, std::string *why)
{
    auto fail = [&](const std::string &m) -> std::unique_ptr<Executor> {
        if (why) *why = m;
        return nullptr;
    };
    std::string reason;
    if (!validate_plan(plan, &reason)) return fail(reason);
    if (in_w < 1 || in_h < 1) return fail("bad input size");
    const int u = plan.unshuffle;
    // the reference's layout check (src/native/layout.cpp:18)
    if (in_w % u || in_h % u) return fail("this model needs even video dimensions");
    std::unique_ptr<Executor> e(new Executor());
    e->U_ = u;
    e->W_ = in_w / u;
    e->H_ = in_h / u;
    e->R_ = plan.depth_to_space;
    in_w = e->W_;
    in_h = e->H_;

    for (size_t i = 0; i < plan.steps.size(); i++) {
        const PlanStep &ps = plan.steps[i];
        Step st;
        st.src = ps.src;
        st.resid = ps.resid;
        st.dst = ps.dst;
        const PlanWeights &pw = ps.w;
        // the head reads the model input packed into a strip-chunked map of 8 (16 unshuffled)
        // channels: its weights gain zero input channels to match
        const bool head = ps.kind == PlanStep::CONV && (ps.in == AJIB_IN_NCHW3 || ps.in == AJIB_IN_NCHW3_UNSHUFFLE2);
        const int cin = head ? (ps.in == AJIB_IN_NCHW3 ? 8 : 16) : pw.cin;
        std::vector<uint16_t> wpad;
        if (head) {
            wpad.assign((size_t)9 * cin * pw.cout, 0);
            for (int t = 0; t < 9; t++)
                for (int k = 0; k < pw.cin; k++)
                    for (int o = 0; o < pw.cout; o++)
                        wpad[((size_t)t * cin + k) * pw.cout + o] = pw.w[((size_t)t * pw.cin + k) * pw.cout + o];
        }
        int rc = ajib_weights_upload(&st.w, head ? wpad.data() : pw.w.data(), pw.bias.data(),
                                     pw.slope.empty() ? nullptr : pw.slope.data(), pw.taps, cin, pw.cout);
        if (rc != AJIB_OK) return fail("weight upload failed (step " + std::to_string(i) + ")");
        if (head) {
            st.pack = true;
            st.pack_c = cin;
            st.unshuffle = ps.in == AJIB_IN_NCHW3_UNSHUFFLE2 ? 1 : 0;
            st.in_norm = ps.in_norm;
            for (int c = 0; c < 3; c++) {
                st.in_mean[c] = ps.in_mean[c];
                st.in_scale[c] = ps.in_scale[c];
            }
            const size_t need = ajib_feature_bytes(in_h, in_w, cin);
            if (cudaMalloc(&st.pack_buf, need) != cudaSuccess || cudaMemset(st.pack_buf, 0, need) != cudaSuccess) {
                cudaFree(st.pack_buf);
                cudaGetLastError();
                ajib_weights_release(&st.w);
                return fail("input buffer allocation failed");
            }
            e->bytes_ += need;
            e->pack_bytes_ = need;
        }
        e->weight_bytes_ += ajib_weights_bytes(st.w);
        if (ps.kind == PlanStep::CONCAT) {
            st.concat = true;
            st.c = ps.c;
            st.nsrc = ps.nsrc;
            for (int k = 0; k < 4; k++) st.srcs[k] = ps.srcs[k];
            e->steps_.push_back(st);
            continue;
        }
        ajib_conv &op = st.op;
        op.in = head ? AJIB_IN_NHWC : ps.in;
        op.act = ps.act;
        op.gate = ps.gate;
        op.out = ps.out;
        op.cin = head ? cin : ps.cin;
        op.cout = ps.cout;
        op.w = st.w;
        if (ps.gate == AJIB_GATE_TANH1X1) {
            const PlanWeights &pa = ps.att;
            if (ajib_weights_upload(&st.att, pa.w.data(), pa.bias.data(), nullptr, pa.taps, pa.cin, pa.cout) != AJIB_OK) {
                ajib_weights_release(&st.w);
                return fail("weight upload failed (step " + std::to_string(i) + ", attention)");
            }
            e->weight_bytes_ += ajib_weights_bytes(st.att);
            op.att = st.att;
        }
        op.in_norm = head ? 0 : ps.in_norm;
        op.out_clamp = ps.out_clamp;
        for (int c = 0; c < 3; c++) {
            op.in_mean[c] = ps.in_mean[c];
            op.in_scale[c] = ps.in_scale[c];
        }
        e->steps_.push_back(st);
        char buf[256] = {0};
        if (!ajib_conv_supported(&e->steps_.back().op, buf, sizeof(buf)))
            return fail("conv " + std::to_string(ps.cin) + "->" + std::to_string(ps.cout) + ": " + buf);
    }

    // feature buffers: a buffer of the same size is reused once its tensor's last reader has run
    const int ns = (int)plan.steps.size(), nt = (int)plan.channels.size();
    std::vector<int> last(nt, -1), born(nt, -1), buffer(nt, -1);
    for (int i = 0; i < ns; i++) {
        const PlanStep &s = plan.steps[i];
        auto read = [&](int t) {
            if (t >= 0) last[t] = i;
        };
        read(s.src);
        read(s.resid);
        if (s.kind == PlanStep::CONCAT)
            for (int t : s.srcs) read(t);
        if (s.dst >= 0) born[s.dst] = i;
    }
    std::vector<size_t> sizes;
    std::vector<std::pair<size_t, int>> free_list;
    for (int i = 0; i < ns; i++) {
        const int d = plan.steps[i].dst;
        if (d >= 0 && buffer[d] < 0) {
            const size_t need = ajib_feature_bytes(in_h, in_w, plan.channels[d]);
            int b = -1;
            for (size_t k = 0; k < free_list.size(); k++)
                if (free_list[k].first == need) {
                    b = free_list[k].second;
                    free_list.erase(free_list.begin() + k);
                    break;
                }
            if (b < 0) {
                b = (int)sizes.size();
                sizes.push_back(need);
            }
            buffer[d] = b;
        }
        for (int t = 0; t < nt; t++)
            if (buffer[t] >= 0 && (last[t] == i || (last[t] < 0 && born[t] == i)))
                free_list.push_back({ajib_feature_bytes(in_h, in_w, plan.channels[t]), buffer[t]});
    }
    e->last_w_ = in_w;
    for (size_t need : sizes) {
        e->buffer_bytes_.push_back(need);
        void *b = nullptr;
        // the image-edge columns of strip-chunked maps must read as zero: clear once, kernels never
        // write them
        if (cudaMalloc(&b, need) != cudaSuccess || cudaMemset(b, 0, need) != cudaSuccess) {
            cudaFree(b);
            cudaGetLastError();
            return fail("feature buffer allocation failed (" + std::to_string(need >> 20) + " MB)");
        }
        e->buffers_.push_back(b);
        e->bytes_ += need;
    }
    e->bytes_ += e->weight_bytes_;
    e->tensor_.assign(nt, nullptr);
    for (int t = 0; t < nt; t++)
        if (buffer[t] >= 0) e->tensor_[t] = e->buffers_[buffer[t]];
    return e;
}

int Executor::profile(bool on)
{
    if (on && prof_ev_.empty()) {
        prof_ev_.assign((size_t)kProfRuns * steps_.size() * 2, nullptr);
        for (cudaEvent_t &e : prof_ev_)
            if (cudaEventCreate(&e) != cudaSuccess) return AJIB_ERR_CUDA;
    }
    prof_on_ = on;
    prof_runs_ = 0;
    return AJIB_OK;
}

int Executor::profile_read(double *ms, int *counts, int nsteps) const
{
    const int ns = (int)steps_.size();
    for (int k = 0; k < nsteps; k++) {
        ms[k] = 0.0;
        counts[k] = 0;
    }
    const int runs = std::min(prof_runs_, kProfRuns);
    for (int r = 0; r < runs; r++)
        for (int k = 0; k < std::min(ns, nsteps); k++) {
            cudaEvent_t a = prof_ev_[((size_t)r * ns + k) * 2], b = prof_ev_[((size_t)r * ns + k) * 2 + 1];
            if (cudaEventSynchronize(b) != cudaSuccess) return AJIB_ERR_CUDA;
            float t = 0.f;
            if (cudaEventElapsedTime(&t, a, b) != cudaSuccess) return AJIB_ERR_CUDA;
            ms[k] += t;
            counts[k]++;
        }
    return AJIB_OK;
}

int Executor::run(const void *in, void *out, int w, int h, cudaStream_t s) const { return run_images(in, out, w, h, 1, s); }

bool Executor::input_pack(InputPack *pk) const
{
    if (steps_.empty() || !steps_[0].pack) return false;
    const Step &st = steps_[0];
    if (pk) {
        pk->map = st.pack_buf;
        pk->unshuffle = st.unshuffle != 0;
        pk->in_norm = st.in_norm;
        for (int c = 0; c < 3; c++) {
            pk->mean[c] = st.in_mean[c];
            pk->scale[c] = st.in_scale[c];
        }
    }
    return true;
}

int Executor::run_packed(const void *in, void *out, cudaStream_t s) const
{
    // the map was written for the whole frame at the created size; a run at another width would
    // first clear the maps (run_images), erasing it
    if (!input_pack(nullptr) || last_w_ != W_) return AJIB_ERR_ARGS;
    return run_steps(in, out, W_ * U_, H_ * U_, 1, s, true);
}

int Executor::launch(const Step &st, const void *in, void *out, int nimg, int img_h, int w, int r0, int r1,
                     cudaStream_t s, bool packed, size_t out_plane) const
{
    if (st.pack && packed) {
        // the producer of the input wrote the head's map already
        return ajib_conv3x3_launch_images(&st.op, st.pack_buf, nullptr, const_cast<void *>(ptr(st.dst, in, out)), nimg,
                                          img_h, w, r0, r1, s);
    }
    if (st.pack) {
        // the input rows the head's rows [r0, r1) read: one-row halos
        const int H = nimg * img_h;
        const int rc = pack_model_input(in, H, w, st.unshuffle, st.in_norm, st.in_mean, st.in_scale, std::max(0, r0 - 1),
                                        std::min(H, r1 + 1), st.pack_buf, s);
        if (rc != AJIB_OK) return rc;
        return ajib_conv3x3_launch_images(&st.op, st.pack_buf, nullptr, const_cast<void *>(ptr(st.dst, in, out)), nimg,
                                          img_h, w, r0, r1, s);
    }
    if (st.concat) {
        const void *srcs[4] = {nullptr, nullptr, nullptr, nullptr};
        for (int k = 0; k < st.nsrc; k++) srcs[k] = ptr(st.srcs[k], in, out);
        return ajib_concat1x1_launch(st.w, st.nsrc, srcs, st.c, const_cast<void *>(ptr(st.dst, in, out)), nimg * img_h, w,
                                     r0, r1, s);
    }
    // the model output's planes may sit inside a larger stack (run_images' out_plane)
    return conv3x3_launch_planes(&st.op, ptr(st.src, in, out), ptr(st.resid, in, out),
                                 const_cast<void *>(ptr(st.dst, in, out)), nimg, img_h, w, r0, r1, s,
                                 st.dst == kModelOutput ? out_plane : 0);
}

int Executor::run_images(const void *in, void *out, int w, int img_h, int nimg, cudaStream_t s, size_t out_plane) const
{
    return run_steps(in, out, w, img_h, nimg, s, false, out_plane);
}

int Executor::run_steps(const void *in, void *out, int w, int img_h, int nimg, cudaStream_t s, bool packed,
                        size_t out_plane) const
{
    if (w < 1 || img_h < 1 || nimg < 1 || w % U_ || img_h % U_ || !in || !out) return AJIB_ERR_ARGS;
    // the conv resolution
    w /= U_;
    img_h /= U_;
    const int h = img_h * nimg;
    if (w > W_ || h > H_) return AJIB_ERR_ARGS;
    // at another width, columns of a strip-chunked map that held pixels may become columns past
    // the image's edge, which must read as zero again
    if (w != last_w_) {
        for (size_t k = 0; k < buffers_.size(); k++)
            if (cudaMemsetAsync(buffers_[k], 0, buffer_bytes_[k], s) != cudaSuccess) return AJIB_ERR_CUDA;
        for (const Step &st : steps_)
            if (st.pack_buf && cudaMemsetAsync(st.pack_buf, 0, pack_bytes_, s) != cudaSuccess) return AJIB_ERR_CUDA;
        last_w_ = w;
    }
    const int ns = (int)steps_.size();
    // profiling brackets whole steps (all of a step's bands), so it runs unbanded
    const bool prof = prof_on_ && !prof_ev_.empty();
    const int slot = prof ? prof_runs_ % kProfRuns : 0;
    if (prof) {
        for (int k = 0; k < ns; k++) {
            const Step &st = steps_[k];
            cudaEventRecord(prof_ev_[((size_t)slot * ns + k) * 2], s);
            const int rc = launch(st, in, out, nimg, img_h, w, 0, h, s, packed, out_plane);
            cudaEventRecord(prof_ev_[((size_t)slot * ns + k) * 2 + 1], s);
            if (rc != AJIB_OK) return rc;
        }
        prof_runs_++;
        return AJIB_OK;
    }
    // band boundaries over the shifted row space [0, h + ns - 1): step k of band b covers rows
    // [B_b - k, B_{b+1} - k) clipped to the frame
    const int nb = std::max(1, std::min(bands_, h));
    for (int b = 0; b < nb; b++) {
        const int span = h + ns - 1;
        const int B0 = (int)((long)span * b / nb), B1 = (int)((long)span * (b + 1) / nb);
        for (int k = 0; k < ns; k++) {
            const Step &st = steps_[k];
            int r0 = nb == 1 ? 0 : std::max(0, B0 - k), r1 = nb == 1 ? h : std::min(h, B1 - k);
            if (r0 >= r1) continue;
            const int rc = launch(st, in, out, nimg, img_h, w, r0, r1, s, packed, out_plane);
            if (rc != AJIB_OK) return rc;
        }
    }
    return AJIB_OK;
}

}  // namespace ajib
