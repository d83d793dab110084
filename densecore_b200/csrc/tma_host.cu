// tma_host.cu -- host-side TMA tensor maps over strided (B, H, rows, D) float32 views.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "tma_host.h"

namespace dc {

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}
}  // namespace

bool tma_stride_ok(int64_t size, int64_t stride) { return size <= 1 || (stride % 4 == 0 && stride > 0); }

// A 4-D map over (D, rows, heads, batch) of a strided float32 tensor; box = 32 x box_rows.
int make_tmap(CUtensorMap *m, const float *base, int64_t D, int64_t rows, int64_t heads, int64_t batch,
              const int64_t *st, int box_rows, CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return fail(DC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    // A size-1 dim's stride is never used; give it a legal value.
    int64_t rs = rows > 1 ? st[2] : 4, hs = heads > 1 ? st[1] : 4, bs = batch > 1 ? st[0] : 4;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)(rows > 0 ? rows : 1), (cuuint64_t)heads, (cuuint64_t)batch};
    cuuint64_t strides[3] = {(cuuint64_t)rs * 4, (cuuint64_t)hs * 4, (cuuint64_t)bs * 4};
    cuuint32_t box[4] = {32, (cuuint32_t)box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DC_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return DC_OK;
}


}  // namespace dc
