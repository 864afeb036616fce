// nd_kv_inst.cuh - instantiates the append and attend kernels for one KV
// element type; included once per nd_kv_*.cu so the four dtypes compile in
// parallel.
#pragma once
#include "nd_internal.h"

namespace nda {

template <typename KVT>
cudaError_t attend_launch_t(int qk, int vd, int nq, const AttnParams &P, dim3 grid, cudaStream_t s) {
#define ND_CASE(Q, V, N)                                                   \
    if (qk == Q && vd == V && nq == N) {                                   \
        attend_kernel<Q, V, KVT, N><<<grid, 128, 0, s>>>(P);               \
        return cudaGetLastError();                                         \
    }
#define ND_CASES(Q, V) ND_CASE(Q, V, 1) ND_CASE(Q, V, 2) ND_CASE(Q, V, 4) ND_CASE(Q, V, 8)
    ND_CASES(48, 64)
    ND_CASES(64, 64)
    ND_CASES(128, 128)
#undef ND_CASES
#undef ND_CASE
    return cudaErrorInvalidValue;
}

template <typename KVT>
cudaError_t append_launch_t(int qk, int vd, const AttnParams &P, cudaStream_t s) {
    const size_t items = (size_t)P.n_tok * P.c.n_kv;
    if (items == 0) return cudaSuccess;
    if constexpr (KvT<KVT>::dt == DT_F16 || KvT<KVT>::dt == DT_BF16) {
        // Vectorised path: no head norm, activations in the cache's type,
        // 16-byte aligned k/v rows.
        const bool vec = !P.knorm && P.act_dt == KvT<KVT>::dt && qk == vd && (qk == 64 || qk == 128) &&
                         ((reinterpret_cast<uintptr_t>(P.k) | reinterpret_cast<uintptr_t>(P.v)) & 15u) == 0;
        if (vec) {
            const size_t rows_per_block = 256 / (qk / 8);
            const unsigned blocks = (unsigned)((items + rows_per_block - 1) / rows_per_block);
            if (qk == 64) append_vec_kernel<64, KVT><<<blocks, 256, 0, s>>>(P);
            else append_vec_kernel<128, KVT><<<blocks, 256, 0, s>>>(P);
            return cudaGetLastError();
        }
    }
    const unsigned blocks = (unsigned)((items + 3) / 4);
#define ND_CASE(Q, V)                                                      \
    if (qk == Q && vd == V) {                                              \
        append_kernel<Q, V, KVT><<<blocks, 128, 0, s>>>(P);                \
        return cudaGetLastError();                                         \
    }
    ND_CASE(48, 64)
    ND_CASE(64, 64)
    ND_CASE(128, 128)
#undef ND_CASE
    return cudaErrorInvalidValue;
}

}  // namespace nda

#define ND_DEFINE_KV(SUF, KVT)                                                                  \
    namespace nda {                                                                             \
    cudaError_t attend_launch_##SUF(int qk, int vd, int nq, const AttnParams &P, dim3 grid,     \
                                    cudaStream_t s) {                                           \
        return attend_launch_t<KVT>(qk, vd, nq, P, grid, s);                                    \
    }                                                                                           \
    cudaError_t append_launch_##SUF(int qk, int vd, const AttnParams &P, cudaStream_t s) {      \
        return append_launch_t<KVT>(qk, vd, P, s);                                              \
    }                                                                                           \
    }
