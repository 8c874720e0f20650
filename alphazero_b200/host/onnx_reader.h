// Reader for the weight container the engine loads: an ONNX ModelProto of
// which only graph initializers are read (the same subset the reference
// loader reads, src/onnx_loader.cpp:88-176):
//   ModelProto.graph (field 7) -> GraphProto.initializer (field 5) ->
//   TensorProto { dims = 1, data_type = 2, float_data = 4, name = 8,
//                 raw_data = 9 }.
// As in the reference, the last graph field wins and, when a name repeats,
// the last tensor of that name wins (src/eigen_engine.cpp:23-25).  Unlike the
// reference, every length is bounds-checked: a truncated or corrupt file
// raises std::runtime_error instead of reading past the buffer.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace mgb {

struct NamedTensor {
    std::string name;
    std::vector<int64_t> dims;
    int data_type = 0;               // ONNX TensorProto.DataType; 1 = FLOAT
    std::vector<float> float_data;   // field 4 (packed or not)
    std::vector<uint8_t> raw_data;   // field 9

    int64_t elements() const;
    // fp32 values: float_data when present, else raw_data read as
    // little-endian fp32 (src/onnx_loader.cpp:74-83).  Throws when the tensor
    // declares a data type other than FLOAT.
    std::vector<float> floats() const;
};

// Parses a serialized ModelProto held in memory.
std::vector<NamedTensor> parse_onnx_initializers(const uint8_t* data, size_t size);

// Reads and parses a file; throws "Cannot open model file: <path>" like the
// reference (src/onnx_loader.cpp:186).
std::vector<NamedTensor> read_onnx_initializers(const std::string& path);

}  // namespace mgb
