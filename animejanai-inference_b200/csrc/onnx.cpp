// onnx.cpp — the protobuf wire-format reader behind parse_onnx (see onnx.h).
//
// Wire format: a message is a sequence of (key, value) with key = field << 3 | wire type; wire
// types 0 varint, 1 fixed64, 2 length-delimited, 5 fixed32. Field numbers of onnx.proto used:
//   ModelProto: graph 7
//   GraphProto: node 1, initializer 5, input 11, output 12
//   NodeProto: input 1, output 2, name 3, op_type 4, attribute 5
//   AttributeProto: name 1, f 2, i 3, s 4, t 5, floats 7, ints 8, type 20
//   TensorProto: dims 1, data_type 2, float_data 4, int32_data 5, int64_data 7, name 8, raw_data 9,
//                double_data 10, data_location 14 (1 = external: refused)
//   ValueInfoProto: name 1
#include "onnx.h"

#include <cstring>
#include <set>

namespace ajib {
namespace {

struct Reader {
    const uint8_t *p, *end;
    bool ok = true;
    Reader(const void *d, size_t n) : p((const uint8_t *)d), end((const uint8_t *)d + n) {}
    bool more() const { return ok && p < end; }
    uint64_t varint()
    {
        uint64_t v = 0;
        for (int shift = 0; shift < 64; shift += 7) {
            if (p >= end) {
                ok = false;
                return 0;
            }
            const uint8_t b = *p++;
            v |= (uint64_t)(b & 0x7f) << shift;
            if (!(b & 0x80)) return v;
        }
        ok = false;
        return 0;
    }
    // a length-delimited field: its bytes
    Reader bytes()
    {
        const uint64_t n = varint();
        if (!ok || n > (uint64_t)(end - p)) {
            ok = false;
            return Reader(p, 0);
        }
        Reader r(p, (size_t)n);
        p += n;
        return r;
    }
    std::string str()
    {
        Reader r = bytes();
        return std::string((const char *)r.p, (size_t)(r.end - r.p));
    }
    uint32_t fixed32()
    {
        if (end - p < 4) {
            ok = false;
            return 0;
        }
        uint32_t v;
        std::memcpy(&v, p, 4);
        p += 4;
        return v;
    }
    uint64_t fixed64()
    {
        if (end - p < 8) {
            ok = false;
            return 0;
        }
        uint64_t v;
        std::memcpy(&v, p, 8);
        p += 8;
        return v;
    }
    void skip(int wt)
    {
        switch (wt) {
        case 0: varint(); break;
        case 1: fixed64(); break;
        case 2: bytes(); break;
        case 5: fixed32(); break;
        default: ok = false;
        }
    }
};

float as_float(uint32_t u)
{
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

bool read_tensor(Reader r, OnnxTensor *t, std::string *why)
{
    std::vector<uint8_t> typed;  // float_data / int32_data / int64_data / double_data, as raw bytes
    bool external = false;
    while (r.more()) {
        const uint64_t key = r.varint();
        const int field = (int)(key >> 3), wt = (int)(key & 7);
        if (field == 1) {  // dims (packed or not)
            if (wt == 2) {
                Reader q = r.bytes();
                while (q.more()) t->dims.push_back((int64_t)q.varint());
                r.ok &= q.ok;
            } else {
                t->dims.push_back((int64_t)r.varint());
            }
        } else if (field == 2 && wt == 0) {
            t->dtype = (int)r.varint();
        } else if (field == 4) {  // float_data: packed fixed32 or single
            if (wt == 2) {
                Reader q = r.bytes();
                typed.insert(typed.end(), q.p, q.end);
            } else {
                const uint32_t u = r.fixed32();
                typed.insert(typed.end(), (const uint8_t *)&u, (const uint8_t *)&u + 4);
            }
        } else if (field == 5 || field == 7) {  // int32_data / int64_data (varints)
            auto put = [&](uint64_t v) {
                if (field == 7) {
                    const int64_t x = (int64_t)v;
                    typed.insert(typed.end(), (const uint8_t *)&x, (const uint8_t *)&x + 8);
                } else {
                    // int32_data also carries float16 / bfloat16 bit patterns (2 bytes) and int32
                    const int32_t x = (int32_t)v;
                    typed.insert(typed.end(), (const uint8_t *)&x, (const uint8_t *)&x + 4);
                }
            };
            if (wt == 2) {
                Reader q = r.bytes();
                while (q.more()) put(q.varint());
                r.ok &= q.ok;
            } else {
                put(r.varint());
            }
        } else if (field == 8 && wt == 2) {
            t->name = r.str();
        } else if (field == 9 && wt == 2) {
            Reader q = r.bytes();
            t->raw.assign(q.p, q.end);
        } else if (field == 10) {  // double_data
            if (wt == 2) {
                Reader q = r.bytes();
                typed.insert(typed.end(), q.p, q.end);
            } else {
                const uint64_t u = r.fixed64();
                typed.insert(typed.end(), (const uint8_t *)&u, (const uint8_t *)&u + 8);
            }
        } else if (field == 14 && wt == 0) {
            external = r.varint() == 1;
        } else {
            r.skip(wt);
        }
    }
    if (!r.ok) {
        *why = "malformed tensor";
        return false;
    }
    if (external) {
        *why = "tensor " + t->name + " uses external data (not supported)";
        return false;
    }
    if (t->raw.empty() && !typed.empty()) {
        if (t->dtype == kOnnxFloat16 || t->dtype == kOnnxBfloat16) {
            // carried as int32 values in int32_data: keep the low 16 bits of each
            for (size_t i = 0; i + 4 <= typed.size(); i += 4) {
                t->raw.push_back(typed[i]);
                t->raw.push_back(typed[i + 1]);
            }
        } else {
            t->raw = std::move(typed);
        }
    }
    return true;
}

bool read_attr(Reader r, OnnxAttr *a, std::string *why)
{
    while (r.more()) {
        const uint64_t key = r.varint();
        const int field = (int)(key >> 3), wt = (int)(key & 7);
        if (field == 1 && wt == 2) {
            a->name = r.str();
        } else if (field == 2 && wt == 5) {
            a->f = as_float(r.fixed32());
        } else if (field == 3 && wt == 0) {
            a->i = (int64_t)r.varint();
        } else if (field == 4 && wt == 2) {
            a->s = r.str();
        } else if (field == 5 && wt == 2) {
            if (!read_tensor(r.bytes(), &a->t, why)) return false;
        } else if (field == 7) {
            if (wt == 2) {
                Reader q = r.bytes();
                while (q.more()) a->floats.push_back(as_float(q.fixed32()));
                r.ok &= q.ok;
            } else {
                a->floats.push_back(as_float(r.fixed32()));
            }
        } else if (field == 8) {
            if (wt == 2) {
                Reader q = r.bytes();
                while (q.more()) a->ints.push_back((int64_t)q.varint());
                r.ok &= q.ok;
            } else {
                a->ints.push_back((int64_t)r.varint());
            }
        } else if (field == 20 && wt == 0) {
            a->type = (int)r.varint();
        } else {
            r.skip(wt);
        }
    }
    if (!r.ok) *why = "malformed attribute";
    return r.ok;
}

bool read_node(Reader r, OnnxNode *n, std::string *why)
{
    while (r.more()) {
        const uint64_t key = r.varint();
        const int field = (int)(key >> 3), wt = (int)(key & 7);
        if (field == 1 && wt == 2) {
            n->in.push_back(r.str());
        } else if (field == 2 && wt == 2) {
            n->out.push_back(r.str());
        } else if (field == 3 && wt == 2) {
            n->name = r.str();
        } else if (field == 4 && wt == 2) {
            n->op = r.str();
        } else if (field == 5 && wt == 2) {
            OnnxAttr a;
            if (!read_attr(r.bytes(), &a, why)) return false;
            n->attrs.push_back(std::move(a));
        } else {
            r.skip(wt);
        }
    }
    if (!r.ok) *why = "malformed node";
    return r.ok;
}

// ValueInfoProto: only its name
std::string value_name(Reader r)
{
    std::string name;
    while (r.more()) {
        const uint64_t key = r.varint();
        if ((key >> 3) == 1 && (key & 7) == 2)
            name = r.str();
        else
            r.skip((int)(key & 7));
    }
    return name;
}

bool read_graph(Reader r, OnnxModel *m, std::string *why)
{
    std::vector<std::string> ins;
    while (r.more()) {
        const uint64_t key = r.varint();
        const int field = (int)(key >> 3), wt = (int)(key & 7);
        if (field == 1 && wt == 2) {
            OnnxNode n;
            if (!read_node(r.bytes(), &n, why)) return false;
            m->nodes.push_back(std::move(n));
        } else if (field == 5 && wt == 2) {
            OnnxTensor t;
            if (!read_tensor(r.bytes(), &t, why)) return false;
            const std::string name = t.name;
            m->inits[name] = std::move(t);
        } else if (field == 11 && wt == 2) {
            ins.push_back(value_name(r.bytes()));
        } else if (field == 12 && wt == 2) {
            m->outputs.push_back(value_name(r.bytes()));
        } else {
            r.skip(wt);
        }
    }
    if (!r.ok) {
        *why = "malformed graph";
        return false;
    }
    // older exporters list initializers among the inputs
    for (const std::string &n : ins)
        if (!m->inits.count(n)) m->inputs.push_back(n);
    return true;
}

}  // namespace

size_t OnnxTensor::count() const
{
    size_t n = 1;
    for (int64_t d : dims) {
        if (d < 0 || d > (int64_t)1 << 28) return 0;
        n *= (size_t)d;
        if (n > (size_t)1 << 28) return 0;
    }
    return n;
}

bool OnnxTensor::to_floats(std::vector<float> *out) const
{
    const size_t n = count();
    out->clear();
    if (dtype == kOnnxFloat && raw.size() == n * 4) {
        out->resize(n);
        if (n) std::memcpy(out->data(), raw.data(), n * 4);
        return true;
    }
    if (dtype == kOnnxDouble && raw.size() == n * 8) {
        for (size_t i = 0; i < n; i++) {
            double d;
            std::memcpy(&d, &raw[i * 8], 8);
            out->push_back((float)d);
        }
        return true;
    }
    if ((dtype == kOnnxFloat16 || dtype == kOnnxBfloat16) && raw.size() == n * 2) {
        for (size_t i = 0; i < n; i++) {
            const uint16_t h = (uint16_t)(raw[2 * i] | raw[2 * i + 1] << 8);
            uint32_t bits;
            if (dtype == kOnnxBfloat16) {
                bits = (uint32_t)h << 16;
            } else {
                // IEEE binary16 -> binary32, exactly
                const uint32_t sign = (uint32_t)(h & 0x8000) << 16, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
                if (exp == 0x1f) {
                    bits = sign | 0x7f800000u | (man << 13);
                } else if (exp != 0) {
                    bits = sign | ((exp + 112) << 23) | (man << 13);
                } else if (man == 0) {
                    bits = sign;
                } else {
                    // subnormal: man * 2^-24, normalised by k left shifts
                    int k = 0;
                    uint32_t m = man;
                    while (!(m & 0x400)) {
                        m <<= 1;
                        k++;
                    }
                    bits = sign | ((uint32_t)(113 - k) << 23) | ((m & 0x3ff) << 13);
                }
            }
            float f;
            std::memcpy(&f, &bits, 4);
            out->push_back(f);
        }
        return true;
    }
    return false;
}

bool OnnxTensor::to_ints(std::vector<int64_t> *out) const
{
    const size_t n = count();
    out->clear();
    if (dtype == kOnnxInt64 && raw.size() == n * 8) {
        out->resize(n);
        if (n) std::memcpy(out->data(), raw.data(), n * 8);
        return true;
    }
    if (dtype == kOnnxInt32 && raw.size() == n * 4) {
        for (size_t i = 0; i < n; i++) {
            int32_t x;
            std::memcpy(&x, &raw[i * 4], 4);
            out->push_back(x);
        }
        return true;
    }
    return false;
}

const OnnxAttr *OnnxNode::attr(const char *n) const
{
    for (const OnnxAttr &a : attrs)
        if (a.name == n) return &a;
    return nullptr;
}

int64_t OnnxNode::attr_i(const char *n, int64_t dflt) const
{
    const OnnxAttr *a = attr(n);
    return a ? a->i : dflt;
}

std::string OnnxNode::attr_s(const char *n, const char *dflt) const
{
    const OnnxAttr *a = attr(n);
    return a ? a->s : std::string(dflt);
}

std::vector<int64_t> OnnxNode::attr_ints(const char *n) const
{
    const OnnxAttr *a = attr(n);
    return a ? a->ints : std::vector<int64_t>();
}

bool parse_onnx(const void *data, size_t size, OnnxModel *out, std::string *why)
{
    *out = OnnxModel();
    Reader r(data, size);
    bool graph = false;
    while (r.more()) {
        const uint64_t key = r.varint();
        const int field = (int)(key >> 3), wt = (int)(key & 7);
        if (field == 7 && wt == 2) {
            if (!read_graph(r.bytes(), out, why)) return false;
            graph = true;
        } else {
            r.skip(wt);
        }
    }
    if (!r.ok || !graph) {
        *why = "not an ONNX model";
        return false;
    }
    return true;
}

}  // namespace ajib
