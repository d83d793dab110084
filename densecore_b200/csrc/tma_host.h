// tma_host.h -- TMA tensor maps for the tensor-core kernels (host side).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace dc {

// Whether a dim of `size` with element stride `stride` can be a TMA global dim (stride a
// multiple of 16 bytes; a size-1 dim's stride is never used).
bool tma_stride_ok(int64_t size, int64_t stride);

// A 4-D tiled map over (D, rows, heads, batch) of a float32 tensor with element strides
// st[0..2] = (batch, head, row) (st[3], the D stride, must be 1); the box is 32 floats
// (128 bytes) by box_rows rows; out-of-range rows read as zero.
int make_tmap(CUtensorMap *m, const float *base, int64_t D, int64_t rows, int64_t heads, int64_t batch,
              const int64_t *st, int box_rows, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

}  // namespace dc
