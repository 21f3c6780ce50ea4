// Minimal stand-ins for the few TensorRT types a plugin's enqueue reads
// (nvinfer1::Dims, DataType, PluginTensorDesc). TensorRT itself is not
// installed here; these carry the same member names and meanings so that an
// enqueue body written against TensorRT compiles unchanged against them.
#pragma once
#include <cstdint>

namespace nvinfer1 {

struct Dims {
  static constexpr int32_t MAX_DIMS{8};
  int32_t nbDims;
  int64_t d[MAX_DIMS];
};

enum class DataType : int32_t { kFLOAT = 0, kHALF = 1, kINT8 = 2, kINT32 = 3 };

enum class TensorFormat : int32_t { kLINEAR = 0 };

struct PluginTensorDesc {
  Dims dims;
  DataType type;
  TensorFormat format;
  float scale;
};

}  // namespace nvinfer1
