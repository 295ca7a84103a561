#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

namespace omni {

struct GatherArgs {
  const void* src;
  int64_t src_stride;  // bytes between rows of src
  void* dst;
  int64_t dst_stride;  // bytes between rows of dst
  const void* parent;  // [rows] int32 or int64
  int parent64;
  int64_t src_rows;
  int64_t row_bytes;
  int* status;
};

cudaError_t launch_gather(const GatherArgs& a, int rows, cudaStream_t stream);

}  // namespace omni
