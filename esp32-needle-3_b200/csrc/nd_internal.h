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

// Warps per CTA of the shared-prefix staging kernel (nd_shared.cuh): two CTAs
// per SM, every lane with all 255 registers for its query row and output.
constexpr int kSharedPrefixWarps = 4;

// Sets the calling thread's nd_attn_last_error() message (printf-style) and
// returns `code`.
int report_error(int code, const char *fmt, ...);

// Rows one attend CTA consumes per loop iteration (a split is a multiple).
int attend_rows_per_iter(int kv_dt, int vd, int nq);

#define ND_DECLARE_KV(SUF)                                                                  \
    cudaError_t attend_launch_##SUF(int qk, int vd, int nq, const AttnParams &P, dim3 grid, \
                                    cudaStream_t s);                                        \
    cudaError_t append_launch_##SUF(int qk, int vd, const AttnParams &P, cudaStream_t s);                \
    cudaError_t attend_lean_launch_##SUF(int hd, int nq, const void *kmap, const void *vmap,            \
                                         const void *ksmap, const void *vsmap, const void *ktmap,        \
                                         const void *vtmap, const LeanTok *tk, const AttnParams &P,      \
                                         int *blocks_per_sm, cudaStream_t s);                            \
    cudaError_t attend_shared_launch_##SUF(int qk, int vd, int nq, const AttnParams &P, uint32_t pseq,  \
                                           uint32_t prows, uint32_t tpc, dim3 grid, int variant,        \
                                           float *part, size_t *smem_bytes, cudaStream_t s);
ND_DECLARE_KV(i8)
ND_DECLARE_KV(f32)
ND_DECLARE_KV(f16)
ND_DECLARE_KV(bf16)
#undef ND_DECLARE_KV

// ---- tcgen05 prefill (nd_prefill_tc.cu) ----------------------------------
// One work item = 128 consecutive query tokens of one sequence for one query
// head; the call's tokens are already appended (K1) and do not wrap the ring.
struct PrefillWork {
    uint32_t seq, tok_base, t0, rows, head, pos0;
};

struct PrefillTcParams {
    const PrefillWork *work;
    uint32_t n_work;
    const float2 *rope;
    const float *qnorm;
    const void *gate;
    void *out;
    int act_dt, out_dt;
    uint32_t n_heads, rep, window;
    const int32_t *btab;        // paged cache: block table [seq][blocks_per_seq], or nullptr
    const int *vbig;            // bf16: the layer's flag (V holds a value f16 cannot represent)
    uint32_t blocks_per_seq, block_shift;   // pages of 2^block_shift (>= 64) slots
    float scale_log2;
    int *err;
};

size_t prefill_tc_smem_bytes();
// qmap/kmap/vmap point to CUtensorMap objects (2D, 16-bit, box 64 x 128,
// 128-byte swizzle) over q [tokens][n_heads*64], and one layer's K and V cache.
// omap: the output [tokens][n_heads*64] (box 64 x 128, f32: 32 x 128); csmap:
// the RoPE table as [max_pos][2][32 floats] (box 32 x 2 x 128, 128-byte
// swizzle). `grid` persistent CTAs walk the P.n_work items.
cudaError_t prefill_tc_launch(bool bf16, const void *qmap, const void *kmap, const void *vmap, const void *omap,
                              const void *csmap, const PrefillTcParams &P, uint32_t grid, cudaStream_t s);

}  // namespace nda
