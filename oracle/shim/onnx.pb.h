// Minimal stand-in for the protoc-generated onnx.pb.h. The reference's
// ir/graph.h only needs the type name onnx::AttributeProto to declare
// Node::attributes; the kernels compiled for the oracle never touch attributes.
// Test infrastructure only (libprotobuf/protoc are not available here).
#pragma once
namespace onnx {
class AttributeProto {};
}  // namespace onnx
