// Tensor-map construction shared by the TMA kernels (implemented in gemm.cu).
#pragma once
#include <cuda.h>

namespace mm {

// fp32 tiled tensor map of rank 2..5 with a 128-byte swizzle: 16-byte chunks
// (K-major operands) or 32-byte chunks when `mn_major` (MN-major tf32 operands).
// dims and box in elements, innermost first; strides[i] (elements) is the
// stride of dims[i + 1]. Returns 0, or nonzero when the driver refuses the map.
int encode_tensor_map(CUtensorMap* map, const float* ptr, int rank, const long long* dims, const long long* strides,
                      const int* box, bool mn_major);

}  // namespace mm
