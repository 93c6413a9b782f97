// Minimal reader of the ONNX protobuf wire format: the subset of ModelProto
// an optimized inferc plan uses (what `inferc optimize` writes through
// RewriteOnnxFromIr, src/cli/main.cpp:200-227, and what the reference's
// loader reads, src/frontend/onnx_loader.cc:103 and onnx_to_ir.cc:86-140):
// the graph's nodes with their attributes, initializers (raw_data or typed
// fields), graph inputs / outputs / value_info, and the opset imports. There
// is no libprotobuf on this host, so the decoder is written against the
// public encoding rules (varint / fixed32 / fixed64 / length-delimited
// fields, packed or unpacked repeated scalars) and onnx.proto's field numbers.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace inferc_dev {
namespace onnx {

// TensorProto.DataType values used here.
enum DataType : int32_t {
  kUndefined = 0,
  kFloat = 1,
  kUint8 = 2,
  kInt8 = 3,
  kInt32 = 6,
  kInt64 = 7,
  kBool = 9,
  kDouble = 11,
};

// AttributeProto.AttributeType values used here.
enum AttrType : int32_t {
  kAttrFloat = 1,
  kAttrInt = 2,
  kAttrString = 3,
  kAttrTensor = 4,
  kAttrFloats = 6,
  kAttrInts = 7,
};

struct TensorProto {
  std::string name;
  int32_t data_type = kUndefined;
  std::vector<int64_t> dims;
  std::string raw_data;
  std::vector<float> float_data;
  std::vector<int32_t> int32_data;
  std::vector<int64_t> int64_data;
  std::vector<double> double_data;
  // Little-endian bytes of the tensor (raw_data, or the typed fields packed).
  std::vector<uint8_t> bytes() const;
  int64_t numel() const;
};

struct Attribute {
  std::string name;
  int32_t type = 0;
  float f = 0.f;
  int64_t i = 0;
  std::string s;
  bool has_t = false;
  TensorProto t;
  std::vector<float> floats;
  std::vector<int64_t> ints;
};

struct Node {
  std::string name, op_type, domain;
  std::vector<std::string> inputs, outputs;
  std::vector<Attribute> attrs;
  const Attribute* attr(const std::string& n) const;
  int64_t attr_int(const std::string& n, int64_t dflt) const;
  float attr_float(const std::string& n, float dflt) const;
  std::vector<int64_t> attr_ints(const std::string& n) const;
};

struct ValueInfo {
  std::string name;
  int32_t elem_type = kUndefined;
  std::vector<int64_t> dims;  // -1 = symbolic / unknown
};

struct Graph {
  std::string name;
  std::vector<Node> nodes;
  std::vector<TensorProto> initializers;
  std::vector<ValueInfo> inputs, outputs, value_info;
};

struct Model {
  int64_t ir_version = 0;
  std::vector<std::pair<std::string, int64_t>> opsets;  // (domain, version)
  std::string producer;
  Graph graph;
};

// Parses a serialized ModelProto; false with a message in *err on malformed
// input (truncated field, bad wire type, lengths past the end).
bool parse_model(const uint8_t* data, size_t len, Model* out, std::string* err);

int64_t dtype_bytes(int32_t dt);  // 0 for types the executor does not handle

}  // namespace onnx
}  // namespace inferc_dev
