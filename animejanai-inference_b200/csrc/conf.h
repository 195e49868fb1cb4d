/*
 * conf.h — animejanai.conf for conf mode (internal): profiles ("slots") of chains, each chain a
 * resolution / fps window and the models to run, each model optionally resized before. The
 * semantics are the reference's (src/aji_conf.cpp, a port of animejanai_config.py):
 *  - INI with [global] and [slot_N] sections; keys are case-insensitive;
 *  - chain_C_min_resolution / max_resolution "WxH" ("" -> 0x0 / infxinf; a 0 component of the
 *    maximum is unbounded); the window compares pixel counts w * h;
 *  - chain_C_min_fps (default 0), chain_C_max_fps (default and 0: unbounded);
 *  - chain_C_model_M_name / _resize_factor_before_upscale (percent, default 100) /
 *    _resize_height_before_upscale (default 0 = none), M = 1 .. number of distinct M;
 *  - chain_C_upscale=no drops the chain's models.
 * Models are <model_dir>/<name>.ajnm (this engine's model file) or else <name>.onnx (lowered to
 * a native plan when loaded). The reference's
 * built-in default profiles (slots 1001+) name its shipped ONNX models and are not provided;
 * temporal-fix models and RIFE settings are parsed into flags that make the chain unsupported
 * (temporal) or report RIFE as inactive.
 */
#pragma once

#include <map>
#include <string>
#include <vector>

namespace ajib {

struct ModelConf {
    std::string name;              // empty: a no-op step
    double resize_factor = 100.0;  // percent, applied before the model
    double resize_height = 0.0;    // fit a 16:9 box of this height before the model (0 = none)
};

struct ChainConf {
    int index = 0;
    double min_px = 0.0, max_px = 1e300, min_fps = 0.0, max_fps = 1e300;
    std::vector<ModelConf> models;
    bool temporal = false;  // a temporal-fix model is configured (not served by this engine)
    bool rife = false;      // RIFE is configured (inactive in this engine)
};

struct SlotConf {
    std::string profile_name = "New Profile";
    std::vector<ChainConf> chains;  // by chain number
};

struct Conf {
    bool logging = true;
    std::map<int, SlotConf> slots;
};

// Read path into *out. A missing file gives an empty configuration (no slots), as the
// reference's lenient reader does; false only for unreadable content (*err).
bool load_conf(const std::string &path, Conf *out, std::string *err);

// The first chain of slot whose pixel and fps windows hold (w, h, fps) and whose model files all
// exist in model_dir; each window match skipped for a missing file adds a line to *skipped.
// nullptr: none (passthrough).
const ChainConf *select_chain(const Conf &conf, int slot, const std::string &model_dir, int w, int h, double fps,
                              std::vector<std::string> *skipped);

// <model_dir>/<name>.ajnm if that file exists, else <model_dir>/<name>.onnx if that one does,
// else the .ajnm path (reported as missing).
std::string model_file(const std::string &model_dir, const std::string &name);

// Size arithmetic of the reference's chain configuration (src/aji_trt.cpp:407-423): round to
// the nearest even integer; fit (w, h) into a box_w x box_h box keeping the aspect ratio, the
// box's width limiting when the frame is wider than 16:9.
int round_even(double v);
void fit_box(int w, int h, double box_w, double box_h, int *ow, int *oh);

}  // namespace ajib
