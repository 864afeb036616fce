// nd_internal.h - launcher interface between the C-ABI host code (nd_attn.cu)
// and the per-KV-dtype kernel translation units (nd_kv_*.cu).
#pragma once
#include <cuda_runtime.h>

#include "nd_device.cuh"

namespace nda {

// Head-dim pairs with compiled kernels, and the GQA widths (query heads per
// KV head, rounded up) each is compiled for.
inline bool head_dims_supported(unsigned qk, unsigned vd) {
    return (qk == 48 && vd == 64) || (qk == 64 && vd == 64) || (qk == 128 && vd == 128);
}
inline int nq_for_rep(unsigned rep) { return rep <= 1 ? 1 : rep <= 2 ? 2 : rep <= 4 ? 4 : 8; }

// Rows one attend CTA consumes per loop iteration (a split is a multiple).
int attend_rows_per_iter(int kv_dt, int vd);

#define ND_DECLARE_KV(SUF)                                                                  \
    cudaError_t attend_launch_##SUF(int qk, int vd, int nq, const AttnParams &P, dim3 grid, \
                                    cudaStream_t s);                                        \
    cudaError_t append_launch_##SUF(int qk, int vd, const AttnParams &P, cudaStream_t s);
ND_DECLARE_KV(i8)
ND_DECLARE_KV(f32)
ND_DECLARE_KV(f16)
ND_DECLARE_KV(bf16)
#undef ND_DECLARE_KV

}  // namespace nda
