/*
 * plan.h — the native model: a conv net as a plan of fused steps, and the executor that runs it
 * at one input size. Host C++ (internal; the C ABI is in include/aji_b200.h).
 *
 * A Plan is what the reference's lowering produces (src/native/lower.h:38-77): conv steps that
 * read a feature map or the NCHW RGB model input and fold their activation, SPAN gate or
 * depth-to-space output, and concat steps (a 1x1 conv over 2-4 feature maps). Feature ids >= 0
 * are NHWC fp16 maps at the conv resolution; kModelInput / kModelOutput are the NCHW fp16 RGB
 * model input and output. Models are read from this engine's model file (model.cpp) until the
 * ONNX lowering lands.
 *
 * The Executor (reference src/native/executor.cpp:23-127) uploads the weights, assigns feature
 * buffers with lifetime reuse (reference src/native/layout.cpp:10-77) and launches one kernel
 * per step on a stream, with no allocation or host synchronisation in a run. Unlike the reference it can
 * run the net as horizontal bands: all steps over band 0, then band 1, ..., each step's rows
 * shifted down by one per step so every row a step reads was written by the previous step of the
 * same or an earlier band. A band's activations stay in L2 between the steps.
 */
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/aji_b200.h"

struct ajib_concat_weights;
struct aji_plan;

namespace ajib {

constexpr int kModelInput = -2, kModelOutput = -3;

struct PlanWeights {
    int taps = 0, cin = 0, cout = 0;
    std::vector<uint16_t> w;   // [taps][cin][cout] fp16 bits
    std::vector<float> bias;   // cout
    std::vector<float> slope;  // cout or empty
};

struct PlanStep {
    enum Kind { CONV = 0, CONCAT = 1 } kind = CONV;
    int in = 0, act = 0, gate = 0, out = 0;
    int cin = 0, cout = 0;
    PlanWeights w, att;
    int src = -1, resid = -1, dst = -1;
    bool in_norm = false;
    float in_mean[3] = {0.f, 0.f, 0.f}, in_scale[3] = {1.f, 1.f, 1.f};
    bool out_clamp = false;
    int c = 0, nsrc = 0;
    int srcs[4] = {-1, -1, -1, -1};
};

struct Plan {
    std::vector<PlanStep> steps;
    std::vector<int> channels;  // per feature id
    int unshuffle = 1;
    int depth_to_space = 1;
    std::string name;
};

// Parse this engine's model file (layout documented in model.cpp). *why on failure.
bool parse_model(const void *data, size_t size, Plan *out, std::string *why);
// A native model file, or an ONNX model file lowered to a plan (lower.cpp).
bool load_model_file(const std::string &path, Plan *out, std::string *why);
bool load_model_bytes(const void *data, size_t size, Plan *out, std::string *why);
// The native model file of a plan.
std::vector<uint8_t> serialize_model(const Plan &p);
struct OnnxModel;
bool lower_onnx(const OnnxModel &m, Plan *plan, std::string *why);
bool validate_plan(const Plan &p, std::string *why);
std::string describe(const Plan &p);
// FLOPs per conv-resolution pixel (algorithmic: 2 * taps * cin * cout per conv output pixel,
// plus 2 * cout * cout for a tanh gate's 1x1 attention).
double flops_per_pixel(const Plan &p);
// The model's scale: output / input size (depth-to-space over pixel-unshuffle).
inline int model_scale(const Plan &p) { return p.depth_to_space / (p.unshuffle > 0 ? p.unshuffle : 1); }

// Where the colour pre pass writes the head conv's input when it is fused with the executor's
// input pack (video.cpp): the head's strip-chunked map (8 channels; with unshuffle, the 16 of the
// 2x pixel-unshuffled input at half size) and the model's input normalisation.
struct InputPack {
    void *map = nullptr;
    bool unshuffle = false;
    bool in_norm = false;
    float mean[3] = {0.f, 0.f, 0.f}, scale[3] = {1.f, 1.f, 1.f};
};

// The NV12 / P010 pre pass (aji_run_pre) writing, besides the NCHW fp16 RGB dst [3][h][w], the
// head's input map pk.map of the same pixels (colour.cu). Returns 0 or a cudaError_t.
int run_pre_packed(aji_plan *p, const void *y_plane, ptrdiff_t y_stride, const void *uv_plane, ptrdiff_t uv_stride,
                   const aji_csp *csp, void *dst_f16, const InputPack &pk, cudaStream_t s);

// The NCHW fp16 model input [3][H][W] (pixel-unshuffled by 2: [3][2H][2W]) of conv rows
// [row_begin, row_end) as a strip-chunked map at H x W of 8 channels {r, g, b, 0...} (16: the 12
// unshuffled channels, then zeros), normalised if in_norm; pad columns untouched (conv.cu).
int pack_model_input(const void *src, int H, int W, int unshuffle, bool in_norm, const float *mean, const float *scale,
                     int row_begin, int row_end, void *dst, cudaStream_t s);

// ajib_conv3x3_launch_images with, for a depth-to-space output, dst_plane elements from one output
// plane to the next (0: the dense [3][R*H][R*W]; else at least one dense plane), so that a batch
// of tiles lands inside a larger stack of tiles (conv.cu).
int conv3x3_launch_planes(const ajib_conv *op, const void *src, const void *resid, void *dst, int nimg, int img_h,
                          int W, int row_begin, int row_end, void *stream, size_t dst_plane);

class Executor {
public:
    static std::unique_ptr<Executor> create(const Plan &plan, int in_w, int in_h, std::string *why);
    ~Executor();
    Executor(const Executor &) = delete;
    Executor &operator=(const Executor &) = delete;

    // the model input size (U times the conv resolution for a pixel-unshuffled input)
    int in_w() const { return W_ * U_; }
    int in_h() const { return H_ * U_; }
    int out_w() const { return W_ * R_; }
    int out_h() const { return H_ * R_; }
    int scale() const { return R_ / U_; }
    size_t device_bytes() const { return bytes_; }
    size_t weight_bytes() const { return weight_bytes_; }
    int launches_per_run() const;
    // launches per run_packed (the head's input pack left to the producer of the input)
    int launches_per_run_packed() const;
    // bands <= 1: one launch per step over the whole frame; else the banded schedule.
    void set_bands(int bands) { bands_ = bands < 1 ? 1 : bands; }
    int bands() const { return bands_; }
    // in: NCHW fp16 [3][h][w], out: NCHW fp16 [3][scale*h][scale*w]; w <= in_w(), h <= in_h(), both
    // multiples of the plan's unshuffle factor.
    int run(const void *in, void *out, int w, int h, cudaStream_t s) const;
    int run(const void *in, void *out, cudaStream_t s) const { return run(in, out, in_w(), in_h(), s); }
    // nimg images of img_h rows each, stacked along H (nimg * img_h <= in_h()), each convolved on
    // its own: in [3][nimg * img_h][w], out [3][scale * nimg * img_h][scale * w], its planes
    // out_plane elements apart when out_plane is not 0 (inside a larger stack of images).
    int run_images(const void *in, void *out, int w, int img_h, int nimg, cudaStream_t s, size_t out_plane = 0) const;
    // The head's input map, when the head reads the NCHW RGB model input (plain or 2x
    // pixel-unshuffled): a producer that writes it (run_pre_packed) lets run_packed skip the
    // head's own pack launch. False for other heads.
    bool input_pack(InputPack *pk) const;
    // run() at the created size with the head's input map already written from `in` (the NCHW
    // input stays needed: a depth-to-space tail adds it).
    int run_packed(const void *in, void *out, cudaStream_t s) const;
    // Step timing: while enabled, every launch is bracketed by CUDA events on its stream (a ring of
    // kProfRuns runs); profile_read synchronises and returns per-step summed milliseconds and
    // counts of the runs recorded since enabling.
    int profile(bool on);
    int profile_read(double *ms, int *counts, int nsteps) const;

private:
    Executor() = default;
    struct Step {
        bool concat = false;
        // the head: the model input is first packed into pack (a strip-chunked map of pack_c
        // channels), which the conv reads by bulk copies like any feature map
        bool pack = false;
        int pack_c = 0, unshuffle = 1;
        bool in_norm = false;
        float in_mean[3] = {0.f, 0.f, 0.f}, in_scale[3] = {1.f, 1.f, 1.f};
        void *pack_buf = nullptr;
        ajib_conv op{};
        ajib_weights *w = nullptr, *att = nullptr;
        int c = 0, nsrc = 0;
        int src = -1, resid = -1, dst = -1;
        int srcs[4] = {-1, -1, -1, -1};
    };
    const void *ptr(int t, const void *in, void *out) const;
    int launch(const Step &st, const void *in, void *out, int nimg, int img_h, int w, int r0, int r1, cudaStream_t s,
               bool packed = false, size_t out_plane = 0) const;
    int run_steps(const void *in, void *out, int w, int img_h, int nimg, cudaStream_t s, bool packed,
                  size_t out_plane = 0) const;
    static constexpr int kProfRuns = 64;
    mutable std::vector<cudaEvent_t> prof_ev_;  // [kProfRuns][steps][2]
    mutable int prof_runs_ = 0;
    bool prof_on_ = false;
    std::vector<Step> steps_;
    std::vector<void *> buffers_;
    std::vector<size_t> buffer_bytes_;
    std::vector<void *> tensor_;
    size_t pack_bytes_ = 0;
    mutable int last_w_ = 0;  // the conv width of the last run (which columns are past the edge)
    int W_ = 0, H_ = 0, R_ = 1, U_ = 1, bands_ = 1;  // conv resolution, depth-to-space, unshuffle
    size_t bytes_ = 0, weight_bytes_ = 0;
};

}  // namespace ajib
