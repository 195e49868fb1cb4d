// conf.cpp — animejanai.conf reading and chain selection (see conf.h).
#include "conf.h"

#include <algorithm>
#include <cctype>
#include <cstdlib>
#include <fstream>
#include <set>
#include <sys/stat.h>

namespace ajib {
namespace {

std::string lowered(std::string s)
{
    for (char &ch : s) ch = (char)std::tolower((unsigned char)ch);
    return s;
}

std::string trimmed(const std::string &s)
{
    const size_t a = s.find_first_not_of(" \t\r\n");
    if (a == std::string::npos) return "";
    return s.substr(a, s.find_last_not_of(" \t\r\n") - a + 1);
}

bool yes(const std::string &v) { return lowered(trimmed(v)) == "yes"; }

// a number; "inf" is unbounded; empty or unparsable gives dflt
double number(const std::string &v, double dflt)
{
    const std::string s = trimmed(v);
    if (s.empty()) return dflt;
    if (lowered(s) == "inf") return 1e300;
    char *end = nullptr;
    const double d = std::strtod(s.c_str(), &end);
    return end == s.c_str() ? dflt : d;
}

void resolution(const std::string &s, double *w, double *h)
{
    const size_t x = lowered(s).find('x');
    if (x == std::string::npos) return;
    *w = number(s.substr(0, x), 0.0);
    *h = number(s.substr(x + 1), 0.0);
}

using Keys = std::map<std::string, std::string>;

std::string key_or(const Keys &k, const std::string &name, const std::string &dflt)
{
    const auto it = k.find(name);
    return it == k.end() ? dflt : it->second;
}

// the distinct positive integers N of keys "<prefix>N..."
std::set<int> indices(const Keys &k, const std::string &prefix)
{
    std::set<int> ids;
    for (const auto &kv : k)
        if (kv.first.compare(0, prefix.size(), prefix) == 0) {
            const int id = std::atoi(kv.first.c_str() + prefix.size());
            if (id > 0) ids.insert(id);
        }
    return ids;
}

ChainConf read_chain(const Keys &k, int index)
{
    ChainConf c;
    c.index = index;
    const std::string p = "chain_" + std::to_string(index) + "_";
    std::string lo = key_or(k, p + "min_resolution", "0x0"), hi = key_or(k, p + "max_resolution", "0x0");
    if (trimmed(lo).empty()) lo = "0x0";
    if (trimmed(hi).empty()) hi = "infxinf";
    double lw = 0, lh = 0, hw = 0, hh = 0;
    resolution(lo, &lw, &lh);
    resolution(hi, &hw, &hh);
    if (hw == 0) hw = 1e300;
    if (hh == 0) hh = 1e300;
    c.min_px = lw * lh;
    c.max_px = hw * hh;
    c.min_fps = number(key_or(k, p + "min_fps", "0"), 0.0);
    c.max_fps = number(key_or(k, p + "max_fps", "inf"), 1e300);
    if (c.max_fps == 0) c.max_fps = 1e300;
    const std::string mp = p + "model_";
    const int nmodels = (int)indices(k, mp).size();
    for (int m = 1; m <= nmodels; m++) {
        const std::string q = mp + std::to_string(m) + "_";
        ModelConf mc;
        mc.name = trimmed(key_or(k, q + "name", ""));
        mc.resize_factor = number(key_or(k, q + "resize_factor_before_upscale", "100"), 100.0);
        mc.resize_height = number(key_or(k, q + "resize_height_before_upscale", "0"), 0.0);
        if (number(key_or(k, q + "frames", "0"), 0.0) > 1) c.temporal = true;
        c.models.push_back(mc);
    }
    if (!yes(key_or(k, p + "upscale", "yes"))) c.models.clear();
    if (!trimmed(key_or(k, p + "temporal_fix_model", "")).empty()) c.temporal = true;
    c.rife = yes(key_or(k, p + "rife", "no"));
    return c;
}

bool file_exists(const std::string &path)
{
    struct stat st;
    return stat(path.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

}  // namespace

int round_even(double v) { return ((int)(v + 0.5)) & ~1; }

void fit_box(int w, int h, double box_w, double box_h, int *ow, int *oh)
{
    if ((double)w / h > 16.0 / 9.0) {
        *ow = round_even(box_w);
        *oh = round_even(box_w * h / w);
    } else {
        *ow = round_even(box_h * w / h);
        *oh = round_even(box_h);
    }
}

std::string model_file(const std::string &model_dir, const std::string &name)
{
    std::string d = model_dir;
    if (!d.empty() && d.back() != '/') d += '/';
    // this engine's model file if there is one, else the ONNX model (lowered when loaded)
    const std::string native = d + name + ".ajnm", onnx = d + name + ".onnx";
    return file_exists(native) || !file_exists(onnx) ? native : onnx;
}

bool load_conf(const std::string &path, Conf *out, std::string *err)
{
    *out = Conf();
    std::ifstream f(path);
    if (!f) return true;
    std::map<std::string, Keys> sections;
    std::string line, cur;
    while (std::getline(f, line)) {
        const std::string t = trimmed(line);
        if (t.empty() || t[0] == ';' || t[0] == '#') continue;
        if (t.front() == '[' && t.back() == ']') {
            cur = lowered(trimmed(t.substr(1, t.size() - 2)));
            sections[cur];
            continue;
        }
        const size_t eq = t.find('=');
        if (eq == std::string::npos || cur.empty()) continue;
        sections[cur][lowered(trimmed(t.substr(0, eq)))] = trimmed(t.substr(eq + 1));
    }
    if (f.bad()) {
        if (err) *err = "cannot read " + path;
        return false;
    }
    const auto g = sections.find("global");
    if (g != sections.end()) out->logging = lowered(key_or(g->second, "logging", "yes")) != "no";
    for (const auto &sec : sections) {
        if (sec.first.compare(0, 5, "slot_") != 0) continue;
        const int slot = std::atoi(sec.first.c_str() + 5);
        SlotConf s;
        s.profile_name = key_or(sec.second, "profile_name", s.profile_name);
        for (int ch : indices(sec.second, "chain_")) s.chains.push_back(read_chain(sec.second, ch));
        out->slots[slot] = s;
    }
    return true;
}

const ChainConf *select_chain(const Conf &conf, int slot, const std::string &model_dir, int w, int h, double fps,
                              std::vector<std::string> *skipped)
{
    const auto it = conf.slots.find(slot);
    if (it == conf.slots.end()) return nullptr;
    const double px = (double)w * h;
    for (const ChainConf &c : it->second.chains) {
        if (!(c.min_px <= px && px <= c.max_px && c.min_fps <= fps && fps <= c.max_fps)) continue;
        std::string missing;
        for (const ModelConf &m : c.models)
            if (!m.name.empty() && !file_exists(model_file(model_dir, m.name))) {
                missing = m.name;
                break;
            }
        if (!missing.empty()) {
            if (skipped)
                skipped->push_back("Chain " + std::to_string(c.index) + " skipped: model not found: " +
                                   model_file(model_dir, missing));
            continue;
        }
        return &c;
    }
    return nullptr;
}

}  // namespace ajib
