// nd_kv_inst.cuh - instantiates the append and attend kernels for one KV
// element type; included once per nd_kv_*.cu so the four dtypes compile in
// parallel.
#pragma once
#include "nd_decode_tma.cuh"
#include "nd_internal.h"
#include "nd_shared.cuh"

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

// Balanced TMA-staged attend (nd_decode_tma.cuh), launched with programmatic
// stream serialization (it may start under the previous kernel's tail; the
// kernel itself waits where it depends on it). With blocks_per_sm set, only
// raises the kernel's dynamic shared memory limit and reports how many CTAs of
// the instantiation one SM holds (no launch); the host asks once per handle
// and instantiation before the first launch. ksmap / vsmap: the int8 scale
// maps (16-bit instantiations take any valid map and ignore it); ktmap /
// vtmap: the same rows as kmap / vmap in 16-row boxes (item tails); tk: the
// call's tokens when they travel as parameters (LeanTok::n = 0 otherwise).
static_assert(6 * sizeof(CUtensorMap) + sizeof(LeanTok) + sizeof(AttnParams) <= 4096,
              "balanced kernel parameters fit the 4 KB parameter space");
template <typename KVT>
cudaError_t attend_lean_launch_t(int hd, int nq, const void *kmap, const void *vmap, const void *ksmap,
                                 const void *vsmap, const void *ktmap, const void *vtmap, const LeanTok *tk,
                                 const AttnParams &P, int *blocks_per_sm, cudaStream_t s) {
    if constexpr (KvT<KVT>::dt == DT_F16 || KvT<KVT>::dt == DT_BF16 || KvT<KVT>::dt == DT_I8) {
#define ND_CASE(H, N)                                                                                   \
        if (hd == H && nq == N) {                                                                       \
            constexpr uint32_t smem = attend_lean_smem_bytes<H, KVT, N>();                              \
            if (blocks_per_sm) { /* once per handle: sets the smem limit on the handle's device */      \
                cudaError_t e = cudaFuncSetAttribute(attend_lean_kernel<H, KVT, N>,                     \
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
                if (e != cudaSuccess) return e;                                                         \
                return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm,                     \
                                                                     attend_lean_kernel<H, KVT, N>, 224, smem); \
            }                                                                                           \
            cudaLaunchConfig_t cfg = {};                                                                \
            cfg.gridDim = dim3(P.n_cta);                                                                \
            cfg.blockDim = dim3(224);                                                                   \
            cfg.dynamicSmemBytes = smem;                                                                \
            cfg.stream = s;                                                                             \
            cudaLaunchAttribute at[1];                                                                  \
            at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;                              \
            at[0].val.programmaticStreamSerializationAllowed = 1;                                       \
            cfg.attrs = at;                                                                             \
            cfg.numAttrs = 1;                                                                           \
            return cudaLaunchKernelEx(&cfg, attend_lean_kernel<H, KVT, N>,                              \
                                      *static_cast<const CUtensorMap *>(kmap),                          \
                                      *static_cast<const CUtensorMap *>(vmap),                          \
                                      *static_cast<const CUtensorMap *>(ksmap),                         \
                                      *static_cast<const CUtensorMap *>(vsmap),                         \
                                      *static_cast<const CUtensorMap *>(ktmap),                         \
                                      *static_cast<const CUtensorMap *>(vtmap), *tk, P);                \
        }
        if constexpr (KvT<KVT>::dt == DT_I8) {
            // int8: query groups of one or two rows (wider groups would cost
            // registers, hence occupancy; they take the exact-grid kernel).
            ND_CASE(64, 1) ND_CASE(64, 2) ND_CASE(128, 1) ND_CASE(128, 2)
        } else {
            ND_CASE(64, 1) ND_CASE(64, 2) ND_CASE(64, 4) ND_CASE(64, 8)
            ND_CASE(128, 1) ND_CASE(128, 2) ND_CASE(128, 4)
        }
#undef ND_CASE
    }
    return cudaErrorInvalidValue;
}

// Shared-prefix decode (nd_shared.cuh): variant 2 (the prefix pass and the
// own-rows pass as two launches, head dims up to 64; `part` holds the (m, l,
// o) of every (token, query head), [n_tok][n_heads][vd + 2] f32) or variant 1
// (lane map throughout, one launch). With smem_bytes set, only reports the
// dynamic shared memory of the staging launch for `prows` rows (no launch);
// cudaErrorInvalidValue when the variant is not built for the shape.
template <typename KVT>
cudaError_t attend_shared_launch_t(int qk, int vd, int nq, const AttnParams &P, uint32_t pseq, uint32_t prows,
                                   uint32_t tpc, dim3 grid, int variant, float *part, size_t *smem_bytes,
                                   cudaStream_t s) {
#define ND_CASE1(Q, V, N)                                                                             \
    if (qk == Q && vd == V && nq == N) {                                                              \
        const size_t smem = shared_smem_bytes<Q, V, KVT, N>(prows);                                   \
        if (smem_bytes) {                                                                             \
            *smem_bytes = smem;                                                                       \
            return cudaSuccess;                                                                       \
        }                                                                                             \
        cudaError_t e = cudaFuncSetAttribute(attend_shared_kernel<Q, V, KVT, N>,                      \
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        if (e != cudaSuccess) return e;                                                               \
        attend_shared_kernel<Q, V, KVT, N><<<grid, 256, smem, s>>>(P, pseq, prows, tpc);              \
        return cudaGetLastError();                                                                    \
    }
#define ND_CASE2(Q, V, N)                                                                             \
    if (qk == Q && vd == V && nq == N) {                                                              \
        const size_t smem = shared2_smem_bytes<Q, V, KVT, N>(prows);                                  \
        if (smem_bytes) {                                                                             \
            *smem_bytes = smem;                                                                       \
            return cudaSuccess;                                                                       \
        }                                                                                             \
        cudaError_t e = cudaFuncSetAttribute(shared_prefix_kernel<Q, V, KVT, N>,                      \
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        if (e != cudaSuccess) return e;                                                               \
        shared_prefix_kernel<Q, V, KVT, N><<<grid, 32 * kSharedPrefixWarps, smem, s>>>(P, pseq, prows, tpc, part); \
        e = cudaGetLastError();                                                                       \
        if (e != cudaSuccess) return e;                                                               \
        const size_t items = (size_t)P.n_tok * P.c.n_kv;                                              \
        shared_own_kernel<Q, V, KVT, N><<<(unsigned)((items + 3) / 4), 128, 0, s>>>(P, prows, part);  \
        return cudaGetLastError();                                                                    \
    }
    if (variant == 2) {
        ND_CASE2(48, 64, 1) ND_CASE2(48, 64, 2) ND_CASE2(48, 64, 4) ND_CASE2(48, 64, 8)
        ND_CASE2(64, 64, 1) ND_CASE2(64, 64, 2) ND_CASE2(64, 64, 4) ND_CASE2(64, 64, 8)
    } else {
        ND_CASE1(48, 64, 1) ND_CASE1(48, 64, 2) ND_CASE1(48, 64, 4) ND_CASE1(48, 64, 8)
        ND_CASE1(64, 64, 1) ND_CASE1(64, 64, 2) ND_CASE1(64, 64, 4) ND_CASE1(64, 64, 8)
        ND_CASE1(128, 128, 1) ND_CASE1(128, 128, 2) ND_CASE1(128, 128, 4) ND_CASE1(128, 128, 8)
    }
#undef ND_CASE1
#undef ND_CASE2
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
    cudaError_t attend_lean_launch_##SUF(int hd, int nq, const void *kmap, const void *vmap,    \
                                         const void *ksmap, const void *vsmap, const void *ktmap,  \
                                         const void *vtmap, const LeanTok *tk, const AttnParams &P, \
                                         int *blocks_per_sm, cudaStream_t s) {                  \
        return attend_lean_launch_t<KVT>(hd, nq, kmap, vmap, ksmap, vsmap, ktmap, vtmap, tk, P, blocks_per_sm, s); \
    }                                                                                           \
    cudaError_t attend_shared_launch_##SUF(int qk, int vd, int nq, const AttnParams &P, uint32_t pseq,  \
                                           uint32_t prows, uint32_t tpc, dim3 grid, int variant,        \
                                           float *part, size_t *smem_bytes, cudaStream_t s) {   \
        return attend_shared_launch_t<KVT>(qk, vd, nq, P, pseq, prows, tpc, grid, variant, part, smem_bytes, s); \
    }                                                                                           \
    }
