// ONNX wire-format decoder (see onnx_model.h). Field numbers follow
// onnx.proto: ModelProto {ir_version 1, producer_name 2, graph 7,
// opset_import 8}; OperatorSetIdProto {domain 1, version 2}; GraphProto
// {node 1, name 2, initializer 5, input 11, output 12, value_info 13};
// NodeProto {input 1, output 2, name 3, op_type 4, attribute 5, domain 7};
// AttributeProto {name 1, f 2, i 3, s 4, t 5, floats 7, ints 8, type 20};
// TensorProto {dims 1, data_type 2, float_data 4, int32_data 5, int64_data 7,
// name 8, raw_data 9, double_data 10}; ValueInfoProto {name 1, type 2};
// TypeProto {tensor_type 1}; TypeProto.Tensor {elem_type 1, shape 2};
// TensorShapeProto {dim 1}; Dimension {dim_value 1, dim_param 2}.
#include "onnx_model.h"

#include <cstring>
#include <stdexcept>

namespace inferc_dev {
namespace onnx {
namespace {

struct ParseError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// A bounded cursor over one message's bytes.
class Reader {
 public:
  Reader(const uint8_t* p, size_t n) : p_(p), end_(p + n) {}
  bool done() const { return p_ >= end_; }

  uint64_t varint() {
    uint64_t v = 0;
    for (int shift = 0; shift < 64; shift += 7) {
      if (p_ >= end_) throw ParseError("truncated varint");
      const uint8_t b = *p_++;
      v |= uint64_t(b & 0x7f) << shift;
      if (!(b & 0x80)) return v;
    }
    throw ParseError("varint longer than 10 bytes");
  }
  uint32_t fixed32() {
    if (end_ - p_ < 4) throw ParseError("truncated fixed32");
    uint32_t v;
    std::memcpy(&v, p_, 4);
    p_ += 4;
    return v;
  }
  uint64_t fixed64() {
    if (end_ - p_ < 8) throw ParseError("truncated fixed64");
    uint64_t v;
    std::memcpy(&v, p_, 8);
    p_ += 8;
    return v;
  }
  Reader sub() {
    const uint64_t n = varint();
    if (n > (uint64_t)(end_ - p_)) throw ParseError("length-delimited field past the end");
    Reader r(p_, (size_t)n);
    p_ += n;
    return r;
  }
  std::string str() {
    Reader r = sub();
    return std::string(reinterpret_cast<const char*>(r.p_), r.end_ - r.p_);
  }
  // (field number, wire type) of the next key.
  std::pair<uint32_t, uint32_t> key() {
    const uint64_t k = varint();
    return {(uint32_t)(k >> 3), (uint32_t)(k & 7)};
  }
  void skip(uint32_t wt) {
    switch (wt) {
      case 0: varint(); break;
      case 1: fixed64(); break;
      case 2: sub(); break;
      case 5: fixed32(); break;
      default: throw ParseError("unsupported wire type " + std::to_string(wt));
    }
  }

 private:
  const uint8_t* p_;
  const uint8_t* end_;
};

float as_float(uint32_t bits) {
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}
double as_double(uint64_t bits) {
  double d;
  std::memcpy(&d, &bits, 8);
  return d;
}

// Repeated scalar fields arrive packed (wire type 2) or one per key.
void read_varints(Reader& r, uint32_t wt, std::vector<int64_t>* out) {
  if (wt == 2) {
    Reader s = r.sub();
    while (!s.done()) out->push_back((int64_t)s.varint());
  } else if (wt == 0) {
    out->push_back((int64_t)r.varint());
  } else {
    throw ParseError("bad wire type for an integer list");
  }
}
void read_floats(Reader& r, uint32_t wt, std::vector<float>* out) {
  if (wt == 2) {
    Reader s = r.sub();
    while (!s.done()) out->push_back(as_float(s.fixed32()));
  } else if (wt == 5) {
    out->push_back(as_float(r.fixed32()));
  } else {
    throw ParseError("bad wire type for a float list");
  }
}

TensorProto parse_tensor(Reader r) {
  TensorProto t;
  while (!r.done()) {
    auto [f, wt] = r.key();
    switch (f) {
      case 1: read_varints(r, wt, &t.dims); break;
      case 2: t.data_type = (int32_t)r.varint(); break;
      case 4: read_floats(r, wt, &t.float_data); break;
      case 5: {
        std::vector<int64_t> v;
        read_varints(r, wt, &v);
        for (int64_t x : v) t.int32_data.push_back((int32_t)x);
        break;
      }
      case 7: read_varints(r, wt, &t.int64_data); break;
      case 8: t.name = r.str(); break;
      case 9: t.raw_data = r.str(); break;
      case 10:
        if (wt == 2) {
          Reader s = r.sub();
          while (!s.done()) t.double_data.push_back(as_double(s.fixed64()));
        } else if (wt == 1) {
          t.double_data.push_back(as_double(r.fixed64()));
        } else {
          throw ParseError("bad wire type for double_data");
        }
        break;
      default: r.skip(wt);
    }
  }
  return t;
}

Attribute parse_attr(Reader r) {
  Attribute a;
  while (!r.done()) {
    auto [f, wt] = r.key();
    switch (f) {
      case 1: a.name = r.str(); break;
      case 2: a.f = as_float(r.fixed32()); break;
      case 3: a.i = (int64_t)r.varint(); break;
      case 4: a.s = r.str(); break;
      case 5: a.t = parse_tensor(r.sub()); a.has_t = true; break;
      case 7: read_floats(r, wt, &a.floats); break;
      case 8: read_varints(r, wt, &a.ints); break;
      case 20: a.type = (int32_t)r.varint(); break;
      default: r.skip(wt);
    }
  }
  return a;
}

Node parse_node(Reader r) {
  Node n;
  while (!r.done()) {
    auto [f, wt] = r.key();
    switch (f) {
      case 1: n.inputs.push_back(r.str()); break;
      case 2: n.outputs.push_back(r.str()); break;
      case 3: n.name = r.str(); break;
      case 4: n.op_type = r.str(); break;
      case 5: n.attrs.push_back(parse_attr(r.sub())); break;
      case 7: n.domain = r.str(); break;
      default: r.skip(wt);
    }
  }
  return n;
}

void parse_shape(Reader r, std::vector<int64_t>* dims) {
  while (!r.done()) {
    auto [f, wt] = r.key();
    if (f != 1) {
      r.skip(wt);
      continue;
    }
    Reader d = r.sub();
    int64_t v = -1;
    while (!d.done()) {
      auto [g, wt2] = d.key();
      if (g == 1) v = (int64_t)d.varint();
      else d.skip(wt2);  // dim_param: symbolic
    }
    dims->push_back(v);
  }
}

ValueInfo parse_value_info(Reader r) {
  ValueInfo v;
  while (!r.done()) {
    auto [f, wt] = r.key();
    if (f == 1) {
      v.name = r.str();
    } else if (f == 2) {  // TypeProto
      Reader tp = r.sub();
      while (!tp.done()) {
        auto [g, wt2] = tp.key();
        if (g != 1) {
          tp.skip(wt2);
          continue;
        }
        Reader tt = tp.sub();  // TypeProto.Tensor
        while (!tt.done()) {
          auto [h, wt3] = tt.key();
          if (h == 1) v.elem_type = (int32_t)tt.varint();
          else if (h == 2) parse_shape(tt.sub(), &v.dims);
          else tt.skip(wt3);
        }
      }
    } else {
      r.skip(wt);
    }
  }
  return v;
}

Graph parse_graph(Reader r) {
  Graph g;
  while (!r.done()) {
    auto [f, wt] = r.key();
    switch (f) {
      case 1: g.nodes.push_back(parse_node(r.sub())); break;
      case 2: g.name = r.str(); break;
      case 5: g.initializers.push_back(parse_tensor(r.sub())); break;
      case 11: g.inputs.push_back(parse_value_info(r.sub())); break;
      case 12: g.outputs.push_back(parse_value_info(r.sub())); break;
      case 13: g.value_info.push_back(parse_value_info(r.sub())); break;
      default: r.skip(wt);
    }
  }
  return g;
}

}  // namespace

int64_t dtype_bytes(int32_t dt) {
  switch (dt) {
    case kFloat: case kInt32: return 4;
    case kInt64: case kDouble: return 8;
    case kUint8: case kInt8: case kBool: return 1;
    default: return 0;
  }
}

int64_t TensorProto::numel() const {
  int64_t n = 1;
  for (int64_t d : dims) n *= d;
  return n;
}

std::vector<uint8_t> TensorProto::bytes() const {
  if (!raw_data.empty()) return std::vector<uint8_t>(raw_data.begin(), raw_data.end());
  const int64_t n = numel();
  std::vector<uint8_t> out((size_t)(n * dtype_bytes(data_type)));
  auto put = [&](const void* src, size_t elem, size_t count) {
    if (count * elem > out.size()) throw std::runtime_error("initializer data longer than dims");
    std::memcpy(out.data(), src, count * elem);
  };
  switch (data_type) {
    case kFloat: put(float_data.data(), 4, float_data.size()); break;
    case kInt64: put(int64_data.data(), 8, int64_data.size()); break;
    case kDouble: put(double_data.data(), 8, double_data.size()); break;
    case kInt32: put(int32_data.data(), 4, int32_data.size()); break;
    case kBool: case kUint8: case kInt8: {  // stored in int32_data, one per element
      if (int32_data.size() > out.size()) throw std::runtime_error("initializer data too long");
      for (size_t i = 0; i < int32_data.size(); ++i) out[i] = (uint8_t)int32_data[i];
      break;
    }
    default: break;
  }
  return out;
}

const Attribute* Node::attr(const std::string& n) const {
  for (const auto& a : attrs)
    if (a.name == n) return &a;
  return nullptr;
}
int64_t Node::attr_int(const std::string& n, int64_t dflt) const {
  const Attribute* a = attr(n);
  return a ? a->i : dflt;
}
float Node::attr_float(const std::string& n, float dflt) const {
  const Attribute* a = attr(n);
  return a ? a->f : dflt;
}
std::vector<int64_t> Node::attr_ints(const std::string& n) const {
  const Attribute* a = attr(n);
  return a ? a->ints : std::vector<int64_t>();
}

bool parse_model(const uint8_t* data, size_t len, Model* out, std::string* err) {
  try {
    Reader r(data, len);
    Model m;
    bool has_graph = false;
    while (!r.done()) {
      auto [f, wt] = r.key();
      switch (f) {
        case 1: m.ir_version = (int64_t)r.varint(); break;
        case 2: m.producer = r.str(); break;
        case 7: m.graph = parse_graph(r.sub()); has_graph = true; break;
        case 8: {
          Reader o = r.sub();
          std::string dom;
          int64_t ver = 0;
          while (!o.done()) {
            auto [g, wt2] = o.key();
            if (g == 1) dom = o.str();
            else if (g == 2) ver = (int64_t)o.varint();
            else o.skip(wt2);
          }
          m.opsets.emplace_back(dom, ver);
          break;
        }
        default: r.skip(wt);
      }
    }
    if (!has_graph) throw ParseError("model has no graph");
    *out = std::move(m);
    return true;
  } catch (const std::exception& e) {
    if (err) *err = e.what();
    return false;
  }
}

}  // namespace onnx
}  // namespace inferc_dev
