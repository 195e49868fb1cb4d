/*
 * onnx.h — an ONNX model file read far enough to lower it to a native plan (internal, host
 * only): the graph's nodes (op, inputs, outputs, attributes), initializers with their data, the
 * graph's inputs and outputs. The file is decoded straight from the protobuf wire format (the
 * public onnx.proto field numbers), with no onnx or protobuf library; external data is not
 * supported. Untrusted input: every length and count is checked against the buffer.
 */
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace ajib {

enum OnnxDtype { kOnnxFloat = 1, kOnnxInt32 = 6, kOnnxInt64 = 7, kOnnxFloat16 = 10, kOnnxDouble = 11, kOnnxBfloat16 = 16 };

struct OnnxTensor {
    std::string name;
    int dtype = 0;
    std::vector<int64_t> dims;
    std::vector<uint8_t> raw;  // little-endian element bytes, from raw_data or the typed fields
    // element count by dims (0 for a bad or huge shape)
    size_t count() const;
    bool to_floats(std::vector<float> *out) const;  // FLOAT, FLOAT16, DOUBLE, BFLOAT16
    bool to_ints(std::vector<int64_t> *out) const;  // INT32, INT64
};

struct OnnxAttr {
    std::string name;
    int type = 0;  // 1 FLOAT, 2 INT, 3 STRING, 4 TENSOR, 6 FLOATS, 7 INTS
    float f = 0.f;
    int64_t i = 0;
    std::string s;
    OnnxTensor t;
    std::vector<float> floats;
    std::vector<int64_t> ints;
};

struct OnnxNode {
    std::string op, name;
    std::vector<std::string> in, out;
    std::vector<OnnxAttr> attrs;
    const OnnxAttr *attr(const char *n) const;
    int64_t attr_i(const char *n, int64_t dflt) const;
    std::string attr_s(const char *n, const char *dflt) const;
    std::vector<int64_t> attr_ints(const char *n) const;
};

struct OnnxModel {
    std::vector<OnnxNode> nodes;
    std::map<std::string, OnnxTensor> inits;
    std::vector<std::string> inputs, outputs;  // graph inputs (initializers excluded) and outputs
};

bool parse_onnx(const void *data, size_t size, OnnxModel *out, std::string *why);

}  // namespace ajib
