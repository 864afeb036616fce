// nd_shared.cuh - decode attention of many sequences whose caches begin with
// the same rows: shared-prefix serving, where every request is restored from
// one saved schema prefix (esp32/main/main.c:281-315 restores it per request;
// nd_model_prefix_restore, engine/src/nd_model.c:1543-1553) and then attends
// to the prefix rows plus its own.
//
// Same results as attend_kernel (nd_device.cuh) for calls in which no
// position wraps the ring (visit index == slot == position): token t at
// position p attends to rows [0, p], the newest (p) appended first (fused K1,
// warp_append). What changes is where the first `prows` rows come from: one
// CTA stages rows [0, prows) of KV head g of the prefix sequence in shared
// memory once and serves many tokens from them, so the prefix is read from L2
// once per CTA instead of once per token. Each token's own rows [prows, p]
// stream from the cache with attend_kernel's lane map.
//
// Two kernels:
//   attend_shared_kernel  (variant 1) the lane map throughout; a warp scores
//                         TB tokens' query rows against each staged row.
//   variant 2 (head dims up to 64): shared_prefix_kernel gives every lane
//                         one (token, query head) pair, its query row and
//                         output accumulator in registers, the staged rows
//                         as f32 broadcast reads, and writes the pair's
//                         (m, l, o); shared_own_kernel (one warp per token
//                         and KV head) continues that softmax over the
//                         token's own rows.
//
// The caller guarantees that rows [0, prows) of every sequence of the call
// hold the prefix sequence's values (shared pages, or prefix_restore from the
// same image); the host checks positions (no wrap, p >= prows, prows written).
#pragma once
#include "nd_internal.h"

namespace nda {

// Tokens per warp (TB) and query rows scored against each staged row
// (NE = TB * NQ), warps per CTA.
template <int NQ>
struct SharedShape {
    static constexpr int TB = NQ >= 4 ? 1 : 4 / NQ;
    static constexpr int NE = TB * NQ;
    static constexpr int NWS = 8;
    static constexpr int MINB = NE >= 8 ? 1 : 2;   // CTAs per SM the register budget is sized for
};

__host__ __device__ constexpr size_t shared_align16(size_t x) { return (x + 15) / 16 * 16; }

// Dynamic shared memory of attend_shared_kernel: the staged K and V rows,
// int8 scales, and per warp its NE query rows in f32.
template <int QK, int VD, typename KVT, int NQ>
__host__ __device__ constexpr size_t shared_smem_bytes(uint32_t prows) {
    return shared_align16((size_t)prows * QK * sizeof(KVT)) + shared_align16((size_t)prows * VD * sizeof(KVT)) +
           (KvT<KVT>::dt == DT_I8 ? 2 * shared_align16((size_t)prows * 4) : 0) +
           (size_t)SharedShape<NQ>::NWS * SharedShape<NQ>::NE * QK * 4;
}

template <int W>
__device__ __forceinline__ void lds_words(const unsigned char *p, uint32_t (&w)[W]) {
    if constexpr (W == 4) {
        const uint4 x = *reinterpret_cast<const uint4 *>(p);
        w[0] = x.x, w[1] = x.y, w[2] = x.z, w[3] = x.w;
    } else if constexpr (W == 2) {
        const uint2 x = *reinterpret_cast<const uint2 *>(p);
        w[0] = x.x, w[1] = x.y;
    } else {
#pragma unroll
        for (int i = 0; i < W; i++) w[i] = reinterpret_cast<const uint32_t *>(p)[i];
    }
}

// grid = (n_kv, ceil(n_tok / tpc)); CTA (g, y) serves tokens [y * tpc,
// (y + 1) * tpc) for KV head g; warp w takes TB consecutive tokens at a time.
template <int QK, int VD, typename KVT, int NQ>
__global__ void __launch_bounds__(256, SharedShape<NQ>::MINB)
    attend_shared_kernel(const AttnParams P, uint32_t pseq, uint32_t prows, uint32_t tpc) {
    using S = AttendShape<QK, VD, KVT, NQ>;   // the lane map of attend_kernel
    constexpr int LPR = S::LPR, RPW = S::RPW, EK = S::EK, EV = S::EV, WK = S::WK, WV = S::WV, ES = S::ES;
    constexpr int TB = SharedShape<NQ>::TB, NE = SharedShape<NQ>::NE, NWS = SharedShape<NQ>::NWS;
    constexpr int U = 2;   // staged row groups per warp iteration
    constexpr bool SCALED = KvT<KVT>::dt == DT_I8;
    extern __shared__ __align__(16) unsigned char sh[];
    unsigned char *sk = sh;
    unsigned char *sv = sk + shared_align16((size_t)prows * QK * ES);
    float *sks = reinterpret_cast<float *>(sv + shared_align16((size_t)prows * VD * ES));
    float *svs = sks + (SCALED ? shared_align16((size_t)prows * 4) / 4 : 0);
    float *sq = svs + (SCALED ? shared_align16((size_t)prows * 4) / 4 : 0);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, sub = lane % LPR, rl = lane / LPR;
    const uint32_t g = blockIdx.x, n_kv = P.c.n_kv, W = P.c.window, rep = P.rep;

    // Rows [0, prows) of KV head g of the prefix sequence, 16-byte chunks.
    {
        constexpr uint32_t KC = QK * ES / 16, VC = VD * ES / 16;
        static_assert((QK * ES) % 16 == 0 && (VD * ES) % 16 == 0, "16-byte row chunks");
        const char *kc = static_cast<const char *>(P.c.k), *vc = static_cast<const char *>(P.c.v);
        for (uint32_t i = tid; i < prows * KC; i += blockDim.x) {
            const uint32_t r = i / KC, c = i - r * KC;
            const size_t row = phys_row(P.c, pseq, r);
            *reinterpret_cast<uint4 *>(sk + (size_t)r * QK * ES + c * 16) =
                *reinterpret_cast<const uint4 *>(kc + (row * P.c.k_dim + (size_t)g * QK) * ES + c * 16);
        }
        for (uint32_t i = tid; i < prows * VC; i += blockDim.x) {
            const uint32_t r = i / VC, c = i - r * VC;
            const size_t row = phys_row(P.c, pseq, r);
            *reinterpret_cast<uint4 *>(sv + (size_t)r * VD * ES + c * 16) =
                *reinterpret_cast<const uint4 *>(vc + (row * P.c.v_dim + (size_t)g * VD) * ES + c * 16);
        }
        if constexpr (SCALED) {
            for (uint32_t r = tid; r < prows; r += blockDim.x) {
                const size_t row = phys_row(P.c, pseq, r);
                sks[r] = P.c.ks[row * n_kv + g];
                svs[r] = P.c.vs[row * n_kv + g];
            }
        }
    }
    __syncthreads();

    float *sqw = sq + (size_t)warp * NE * QK;
    const char *kbase = static_cast<const char *>(P.c.k) + ((size_t)g * QK + (size_t)sub * EK) * ES;
    const char *vbase = static_cast<const char *>(P.c.v) + ((size_t)g * VD + (size_t)sub * EV) * ES;
    const size_t krow_bytes = (size_t)P.c.k_dim * ES, vrow_bytes = (size_t)P.c.v_dim * ES;
    const uint32_t t0 = blockIdx.y * tpc;

    for (uint32_t tb = (uint32_t)warp * TB; tb < tpc; tb += NWS * TB) {
        uint32_t seq[TB], pos[TB], orow[TB];
        bool live[TB];
#pragma unroll
        for (int b = 0; b < TB; b++) {
            const uint32_t tok = t0 + tb + b;
            live[b] = tb + b < tpc && tok < P.n_tok;
            seq[b] = pos[b] = orow[b] = 0;
            if (live[b]) {
                const TokMeta tm = token_meta(P, tok);
                const SeqState st = P.state[tm.seq];
                const uint32_t p = st.pos + tm.off;
                if (p >= P.max_pos || p >= W || p < prows || st.n_sink >= W) {
                    if (lane == 0) set_err(P.err, 2);
                    live[b] = false;
                } else {
                    seq[b] = tm.seq, pos[b] = p, orow[b] = tm.row;
                }
            }
        }
        // Query rows (norm + RoPE, log2-domain scale) of the TB tokens, and
        // the append of each token's newest row (only this warp reads it).
#pragma unroll
        for (int b = 0; b < TB; b++) {
            const float2 *cs = P.rope + (size_t)pos[b] * (QK / 2);
#pragma unroll
            for (int qi = 0; qi < NQ; qi++) {
                float *dst = sqw + (b * NQ + qi) * QK;
                if (live[b] && (uint32_t)qi < rep) {
                    RopePairs<QK> x;
                    warp_load_pairs<QK>(x, P.q, P.act_dt, ((size_t)orow[b] * P.n_heads + g * rep + qi) * QK, lane);
                    warp_norm_rope<QK>(x, cs, P.qnorm, lane);
#pragma unroll
                    for (int c = 0; c < RopePairs<QK>::PPL; c++) {
                        const int i = lane + 32 * c;
                        if (i < QK / 2) {
                            dst[i] = x.a[c] * P.scale_log2;
                            dst[i + QK / 2] = x.b[c] * P.scale_log2;
                        }
                    }
                } else {
                    for (int i = lane; i < QK; i += 32) dst[i] = 0.0f;
                }
            }
            if (live[b])
                warp_append<QK, VD, KVT>(P.c, phys_row(P.c, seq[b], pos[b]), g, P.k, P.v, P.act_dt,
                                         ((size_t)orow[b] * n_kv + g) * QK, ((size_t)orow[b] * n_kv + g) * VD, cs,
                                         P.knorm, lane);
        }
        __syncwarp();
        float qr[NE][EK];
#pragma unroll
        for (int e = 0; e < NE; e++)
#pragma unroll
            for (int i = 0; i < EK; i++) qr[e][i] = sqw[e * QK + sub * EK + i];
        __syncwarp();   // sqw is rewritten by the warp's next tokens

        float m[NE], l[NE], acc[NE][EV];
#pragma unroll
        for (int e = 0; e < NE; e++) {
            m[e] = -INFINITY;
            l[e] = 0.0f;
#pragma unroll
            for (int i = 0; i < EV; i++) acc[e][i] = 0.0f;
        }

        // The staged prefix rows, each scored against all NE query rows.
        for (uint32_t base = 0; base < prows; base += U * RPW) {
            uint32_t kw[U][WK], vw[U][WV];
            float ksc[U], vsc[U];
            bool valid[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const uint32_t j = base + u * RPW + rl;
                valid[u] = j < prows;
                const uint32_t jj = valid[u] ? j : 0u;
                lds_words<WK>(sk + (size_t)jj * QK * ES + (size_t)sub * EK * ES, kw[u]);
                lds_words<WV>(sv + (size_t)jj * VD * ES + (size_t)sub * EV * ES, vw[u]);
                ksc[u] = SCALED ? sks[jj] : 0.0f;
                vsc[u] = SCALED ? svs[jj] : 0.0f;
            }
            consume<QK, VD, KVT, NE, U>(qr, kw, vw, ksc, vsc, valid, m, l, acc);
        }

        // Each token's own rows [prows, pos) from the cache, two of the
        // warp's tokens per load round, then its newest row, which this warp
        // wrote above: read back through the coherent path.
        uint32_t own = 0;
#pragma unroll
        for (int b = 0; b < TB; b++) own = max(own, live[b] ? pos[b] - prows + 1 : 0u);
        constexpr int OB = TB < 2 ? TB : 2;   // tokens per load round (registers)
        for (uint32_t i0 = 0; i0 < own; i0 += RPW) {
#pragma unroll
            for (int b0 = 0; b0 < TB; b0 += OB) {
                uint32_t kw[OB][WK], vw[OB][WV];
                float ksc[OB], vsc[OB];
                bool valid[OB];
#pragma unroll
                for (int bb = 0; bb < OB; bb++) {
                    const int b = b0 + bb;
                    const uint32_t j = prows + i0 + rl;
                    valid[bb] = live[b] && j <= pos[b];
                    ksc[bb] = vsc[bb] = 0.0f;
                    if (valid[bb]) {
                        const size_t row = phys_row(P.c, seq[b], j);
                        if (j < pos[b]) {
                            load_words<WK, true>(kbase + row * krow_bytes, kw[bb]);
                            load_words<WV, true>(vbase + row * vrow_bytes, vw[bb]);
                        } else {
                            load_words<WK, false>(kbase + row * krow_bytes, kw[bb]);
                            load_words<WV, false>(vbase + row * vrow_bytes, vw[bb]);
                        }
                        if constexpr (SCALED) {
                            ksc[bb] = P.c.ks[row * n_kv + g];
                            vsc[bb] = P.c.vs[row * n_kv + g];
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < WK; i++) kw[bb][i] = 0u;
#pragma unroll
                        for (int i = 0; i < WV; i++) vw[bb][i] = 0u;
                    }
                }
#pragma unroll
                for (int bb = 0; bb < OB; bb++) {
                    const int b = b0 + bb;
                    float qb[NQ][EK], mb[NQ], lb[NQ], ab[NQ][EV];
                    uint32_t kb[1][WK], vb[1][WV];
                    const float kscb[1] = {ksc[bb]}, vscb[1] = {vsc[bb]};
                    const bool vb1[1] = {valid[bb]};
#pragma unroll
                    for (int i = 0; i < WK; i++) kb[0][i] = kw[bb][i];
#pragma unroll
                    for (int i = 0; i < WV; i++) vb[0][i] = vw[bb][i];
#pragma unroll
                    for (int qi = 0; qi < NQ; qi++) {
                        mb[qi] = m[b * NQ + qi];
                        lb[qi] = l[b * NQ + qi];
#pragma unroll
                        for (int i = 0; i < EK; i++) qb[qi][i] = qr[b * NQ + qi][i];
#pragma unroll
                        for (int i = 0; i < EV; i++) ab[qi][i] = acc[b * NQ + qi][i];
                    }
                    consume<QK, VD, KVT, NQ, 1>(qb, kb, vb, kscb, vscb, vb1, mb, lb, ab);
#pragma unroll
                    for (int qi = 0; qi < NQ; qi++) {
                        m[b * NQ + qi] = mb[qi];
                        l[b * NQ + qi] = lb[qi];
#pragma unroll
                        for (int i = 0; i < EV; i++) acc[b * NQ + qi][i] = ab[qi][i];
                    }
                }
            }
        }

        // The row groups' sums meet (m is warp-uniform), then lanes of row
        // group 0 write their EV output elements of each query row.
#pragma unroll
        for (int e = 0; e < NE; e++) {
#pragma unroll
            for (int o = LPR; o < 32; o <<= 1) {
                l[e] += __shfl_xor_sync(0xffffffffu, l[e], o);
#pragma unroll
                for (int i = 0; i < EV; i++) acc[e][i] += __shfl_xor_sync(0xffffffffu, acc[e][i], o);
            }
        }
#pragma unroll
        for (int b = 0; b < TB; b++) {
#pragma unroll
            for (int qi = 0; qi < NQ; qi++) {
                if (!live[b] || (uint32_t)qi >= rep || rl != 0) continue;
                const int e = b * NQ + qi;
                const uint32_t h = g * rep + qi;
                const size_t ob = ((size_t)orow[b] * P.n_heads + h) * VD;
                const float inv = 1.0f / l[e];
#pragma unroll
                for (int i = 0; i < EV; i++) {
                    const uint32_t d = sub * EV + i;
                    float val = acc[e][i] * inv;
                    if (P.gate)
                        val *= 1.0f / (1.0f + ex2(-act_load(P.gate, P.act_dt, ob + d) * 1.4426950408889634f));
                    out_store<VD>(P, orow[b], h * VD + d, val);
                }
            }
        }
    }
}

// ---- head dims up to 64: the prefix pass as its own kernel
//
// The lane map spends most of its instructions on the lanes' shuffles and the
// per-row softmax upkeep, which a prefix scored by many requests does not
// need. Variant 2 splits the call in two launches:
//   shared_prefix_kernel  every lane takes one (token, query head) pair: its
//                         rotated query row and output accumulator live in
//                         the lane's registers, each staged prefix row (f32,
//                         int8 already scaled) is a broadcast shared-memory
//                         read, and the lane runs its own online softmax over
//                         chunks of 8 rows (one rescale per chunk). It writes
//                         the pair's (m, l, o) over the prefix to `part`.
//   shared_own_kernel     one warp per (token, KV head), many CTAs per SM:
//                         the newest row's append, then attend_kernel's lane
//                         map over the token's own rows [prows, pos], the
//                         softmax seeded with the pair's (m, l, o); output.

template <int QK, int VD, typename KVT, int NQ>
__host__ __device__ constexpr size_t shared2_smem_bytes(uint32_t prows) {
    return (size_t)prows * (QK + VD) * 4;
}

// QK activation values of one head row into f32 registers (16-byte loads).
template <int QK>
__device__ __forceinline__ void lane_load_row(float (&x)[QK], const void *src, int dt, size_t base) {
    if (dt == DT_F32) {
        const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(src) + base);
#pragma unroll
        for (int i = 0; i < QK / 4; i++) {
            const float4 v = p[i];
            x[4 * i] = v.x, x[4 * i + 1] = v.y, x[4 * i + 2] = v.z, x[4 * i + 3] = v.w;
        }
    } else {
        const uint4 *p = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(src) + base);
#pragma unroll
        for (int i = 0; i < QK / 8; i++) {
            const uint4 v = p[i];
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float2 f;
                if (dt == DT_F16) {
                    __half2 h;
                    memcpy(&h, &w[e], 4);
                    f = __half22float2(h);
                } else {
                    f = make_float2(__uint_as_float(w[e] << 16), __uint_as_float(w[e] & 0xffff0000u));
                }
                x[8 * i + 2 * e] = f.x, x[8 * i + 2 * e + 1] = f.y;
            }
        }
    }
}

// Position of token `tok` of the call when it may be served (no wrap, past
// the prefix), else false (and the status word is set).
__device__ __forceinline__ bool shared_token(const AttnParams &P, uint32_t tok, uint32_t prows, TokMeta &tm,
                                             uint32_t &pos) {
    tm = token_meta(P, tok);
    const SeqState st = P.state[tm.seq];
    pos = st.pos + tm.off;
    return !(pos >= P.max_pos || pos >= P.c.window || pos < prows || st.n_sink >= P.c.window);
}

// grid = (n_kv, ceil(n_tok / tpc)); part: [n_tok][n_heads][VD + 2] f32 =
// (m, l, o) of every (token, query head) over the prefix rows.
template <int QK, int VD, typename KVT, int NQ>
__global__ void __launch_bounds__(128, 2)
    shared_prefix_kernel(const AttnParams P, uint32_t pseq, uint32_t prows, uint32_t tpc, float *part) {
    constexpr int NWS = kSharedPrefixWarps, TW = 32 / NQ;
    constexpr bool SCALED = KvT<KVT>::dt == DT_I8;
    static_assert(QK <= 64 && VD <= 64 && QK % 8 == 0 && VD % 4 == 0, "registers per lane");
    extern __shared__ __align__(16) unsigned char sh[];
    float *sK = reinterpret_cast<float *>(sh);             // [prows][QK]
    float *sV = sK + (size_t)prows * QK;                     // [prows][VD]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t g = blockIdx.x, n_kv = P.c.n_kv, rep = P.rep;

    // Rows [0, prows) of KV head g of the prefix sequence as f32 (int8 rows
    // times their scales), 16-byte chunks of the cache rows.
    {
        constexpr int ES = (int)sizeof(KVT), EPC = 16 / ES;   // elements per chunk
        constexpr uint32_t KC = QK * ES / 16, VC = VD * ES / 16;
        static_assert((QK * ES) % 16 == 0 && (VD * ES) % 16 == 0 && EPC % 4 == 0, "16-byte row chunks");
        const char *kc = static_cast<const char *>(P.c.k), *vc = static_cast<const char *>(P.c.v);
#pragma unroll 4
        for (uint32_t i = tid; i < prows * (KC + VC); i += blockDim.x) {
            const bool isk = i < prows * KC;
            const uint32_t ii = isk ? i : i - prows * KC, CPR = isk ? KC : VC;
            const uint32_t r = ii / CPR, c = ii - r * CPR;
            const size_t row = phys_row(P.c, pseq, r);
            const char *src = isk ? kc + (row * P.c.k_dim + (size_t)g * QK) * ES + c * 16
                                  : vc + (row * P.c.v_dim + (size_t)g * VD) * ES + c * 16;
            uint32_t w[4];
            load_words<4, true>(src, w);
            float f[EPC];
            unpack<KVT, 4>(w, f);
            float sc = 1.0f;
            if constexpr (SCALED) sc = isk ? P.c.ks[row * n_kv + g] : P.c.vs[row * n_kv + g];
            float4 *dst = reinterpret_cast<float4 *>((isk ? sK + (size_t)r * QK : sV + (size_t)r * VD) + c * EPC);
#pragma unroll
            for (int e = 0; e < EPC / 4; e++)
                dst[e] = make_float4(f[4 * e] * sc, f[4 * e + 1] * sc, f[4 * e + 2] * sc, f[4 * e + 3] * sc);
        }
    }
    __syncthreads();

    const uint32_t t0 = blockIdx.y * tpc;
    for (uint32_t c0 = (uint32_t)warp * TW; c0 < tpc; c0 += NWS * TW) {
        // lane = (token c0 + lane / NQ, query head g * rep + lane % NQ)
        const uint32_t tl = c0 + lane / NQ, qi = lane % NQ, tok = t0 + tl;
        TokMeta tm{};
        uint32_t pos = 0;
        const bool live = tl < tpc && tok < P.n_tok && qi < rep && shared_token(P, tok, prows, tm, pos);
        float q[QK];
#pragma unroll
        for (int i = 0; i < QK; i++) q[i] = 0.0f;
        if (live) {
            lane_load_row<QK>(q, P.q, P.act_dt, ((size_t)tm.row * P.n_heads + g * rep + qi) * QK);
            if (P.qnorm) {
                float ss = 0.0f;
#pragma unroll
                for (int i = 0; i < QK; i++) ss = fmaf(q[i], q[i], ss);
                const float inv = rsqrtf(ss * (1.0f / QK) + 1e-6f);
#pragma unroll
                for (int i = 0; i < QK; i++) q[i] *= (1.0f + P.qnorm[i]) * inv;
            }
            const float4 *cs4 = reinterpret_cast<const float4 *>(P.rope + (size_t)pos * (QK / 2));
#pragma unroll
            for (int i = 0; i < QK / 2; i += 2) {
                const float4 t = cs4[i / 2];   // pairs i and i + 1: (cos, sin, cos, sin)
                const float a0 = q[i], b0 = q[i + QK / 2], a1 = q[i + 1], b1 = q[i + 1 + QK / 2];
                q[i] = (a0 * t.x - b0 * t.y) * P.scale_log2;
                q[i + QK / 2] = (b0 * t.x + a0 * t.y) * P.scale_log2;
                q[i + 1] = (a1 * t.z - b1 * t.w) * P.scale_log2;
                q[i + 1 + QK / 2] = (b1 * t.z + a1 * t.w) * P.scale_log2;
            }
        }
        float m = -INFINITY, l = 0.0f, o[VD];
#pragma unroll
        for (int i = 0; i < VD; i++) o[i] = 0.0f;
        for (uint32_t k0 = 0; k0 < prows; k0 += 8) {
            // Eight independent dot products, advanced together one 4-wide
            // chunk of the head dim at a time (eight FMA chains in flight).
            float s[8];
            const float4 *kr[8];
#pragma unroll
            for (int kk = 0; kk < 8; kk++) {
                s[kk] = 0.0f;
                kr[kk] = reinterpret_cast<const float4 *>(sK + (size_t)(k0 + kk < prows ? k0 + kk : prows - 1) * QK);
            }
#pragma unroll
            for (int i = 0; i < QK / 4; i++) {
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const float4 kv = kr[kk][i];
                    s[kk] = fmaf(q[4 * i], kv.x, s[kk]);
                    s[kk] = fmaf(q[4 * i + 1], kv.y, s[kk]);
                    s[kk] = fmaf(q[4 * i + 2], kv.z, s[kk]);
                    s[kk] = fmaf(q[4 * i + 3], kv.w, s[kk]);
                }
            }
#pragma unroll
            for (int kk = 0; kk < 8; kk++) s[kk] = k0 + kk < prows ? s[kk] : -INFINITY;
            float mx = s[0];
#pragma unroll
            for (int kk = 1; kk < 8; kk++) mx = fmaxf(mx, s[kk]);
            const float mn = fmaxf(m, mx);
            const float alpha = ex2(m - mn);
            m = mn;
            l *= alpha;
#pragma unroll
            for (int i = 0; i < VD; i++) o[i] *= alpha;
#pragma unroll
            for (int kk = 0; kk < 8; kk++) {
                const uint32_t key = k0 + kk < prows ? k0 + kk : prows - 1;
                const float p = ex2(s[kk] - mn);
                l += p;
                const float4 *vr = reinterpret_cast<const float4 *>(sV + (size_t)key * VD);
#pragma unroll
                for (int i = 0; i < VD / 4; i++) {
                    const float4 vv = vr[i];
                    o[4 * i] = fmaf(p, vv.x, o[4 * i]);
                    o[4 * i + 1] = fmaf(p, vv.y, o[4 * i + 1]);
                    o[4 * i + 2] = fmaf(p, vv.z, o[4 * i + 2]);
                    o[4 * i + 3] = fmaf(p, vv.w, o[4 * i + 3]);
                }
            }
        }
        if (live) {
            float *hp = part + ((size_t)tok * P.n_heads + g * rep + qi) * (VD + 2);
            hp[0] = m;
            hp[1] = l;
#pragma unroll
            for (int i = 0; i < VD; i++) hp[2 + i] = o[i];
        }
    }
}

// One warp per (token, KV head) item; 4 warps per CTA.
template <int QK, int VD, typename KVT, int NQ>
__global__ void __launch_bounds__(128) shared_own_kernel(const AttnParams P, uint32_t prows, const float *part) {
    using S = AttendShape<QK, VD, KVT, NQ>;
    constexpr int LPR = S::LPR, RPW = S::RPW, EK = S::EK, EV = S::EV, WK = S::WK, WV = S::WV, ES = S::ES;
    constexpr int U = 4;   // row groups per iteration (8: 123 registers, 1.69 against 1.49 ms per config-5 step)
    constexpr bool SCALED = KvT<KVT>::dt == DT_I8;
    __shared__ float sq[4][NQ][QK];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, sub = lane % LPR, rl = lane / LPR;
    const uint32_t n_kv = P.c.n_kv, rep = P.rep;
    const size_t item = (size_t)blockIdx.x * 4 + warp;
    if (item >= (size_t)P.n_tok * n_kv) return;
    const uint32_t tok = (uint32_t)(item / n_kv), g = (uint32_t)(item % n_kv);
    TokMeta tm;
    uint32_t pos;
    if (!shared_token(P, tok, prows, tm, pos)) {
        if (lane == 0) set_err(P.err, 2);
        return;
    }
    const float2 *cs = P.rope + (size_t)pos * (QK / 2);
    float *sqw = &sq[warp][0][0];
#pragma unroll
    for (int qi = 0; qi < NQ; qi++) {
        if ((uint32_t)qi < rep) {
            RopePairs<QK> x;
            warp_load_pairs<QK>(x, P.q, P.act_dt, ((size_t)tm.row * P.n_heads + g * rep + qi) * QK, lane);
            warp_norm_rope<QK>(x, cs, P.qnorm, lane);
#pragma unroll
            for (int c = 0; c < RopePairs<QK>::PPL; c++) {
                const int i = lane + 32 * c;
                if (i < QK / 2) {
                    sqw[qi * QK + i] = x.a[c] * P.scale_log2;
                    sqw[qi * QK + i + QK / 2] = x.b[c] * P.scale_log2;
                }
            }
        } else {
            for (int i = lane; i < QK; i += 32) sqw[qi * QK + i] = 0.0f;
        }
    }
    warp_append<QK, VD, KVT>(P.c, phys_row(P.c, tm.seq, pos), g, P.k, P.v, P.act_dt,
                             ((size_t)tm.row * n_kv + g) * QK, ((size_t)tm.row * n_kv + g) * VD, cs, P.knorm, lane);
    __syncwarp();
    float qr[NQ][EK], m[NQ], l[NQ], acc[NQ][EV];
#pragma unroll
    for (int qi = 0; qi < NQ; qi++) {
#pragma unroll
        for (int e = 0; e < EK; e++) qr[qi][e] = sqw[qi * QK + sub * EK + e];
        if ((uint32_t)qi < rep) {
            const float *hp = part + ((size_t)tok * P.n_heads + g * rep + qi) * (VD + 2);
            m[qi] = hp[0];
            l[qi] = rl == 0 ? hp[1] : 0.0f;
#pragma unroll
            for (int e = 0; e < EV; e++) acc[qi][e] = rl == 0 ? hp[2 + sub * EV + e] : 0.0f;
        } else {
            m[qi] = -INFINITY;
            l[qi] = 0.0f;
#pragma unroll
            for (int e = 0; e < EV; e++) acc[qi][e] = 0.0f;
        }
    }
    const char *kbase = static_cast<const char *>(P.c.k) + ((size_t)g * QK + (size_t)sub * EK) * ES;
    const char *vbase = static_cast<const char *>(P.c.v) + ((size_t)g * VD + (size_t)sub * EV) * ES;
    const size_t krow_bytes = (size_t)P.c.k_dim * ES, vrow_bytes = (size_t)P.c.v_dim * ES;
    for (uint32_t base = prows; base <= pos; base += U * RPW) {
        uint32_t kw[U][WK], vw[U][WV];
        float ksc[U], vsc[U];
        bool valid[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const uint32_t j = base + u * RPW + rl;
            valid[u] = j <= pos;
            ksc[u] = vsc[u] = 0.0f;
            if (valid[u]) {
                const size_t row = phys_row(P.c, tm.seq, j);
                if (j < pos) {
                    load_words<WK, true>(kbase + row * krow_bytes, kw[u]);
                    load_words<WV, true>(vbase + row * vrow_bytes, vw[u]);
                } else {   // the newest row, written by this warp: the coherent path
                    load_words<WK, false>(kbase + row * krow_bytes, kw[u]);
                    load_words<WV, false>(vbase + row * vrow_bytes, vw[u]);
                }
                if constexpr (SCALED) {
                    ksc[u] = P.c.ks[row * n_kv + g];
                    vsc[u] = P.c.vs[row * n_kv + g];
                }
            } else {
#pragma unroll
                for (int i = 0; i < WK; i++) kw[u][i] = 0u;
#pragma unroll
                for (int i = 0; i < WV; i++) vw[u][i] = 0u;
            }
        }
        consume<QK, VD, KVT, NQ, U>(qr, kw, vw, ksc, vsc, valid, m, l, acc);
    }
#pragma unroll
    for (int qi = 0; qi < NQ; qi++) {
#pragma unroll
        for (int o = LPR; o < 32; o <<= 1) {
            l[qi] += __shfl_xor_sync(0xffffffffu, l[qi], o);
#pragma unroll
            for (int e = 0; e < EV; e++) acc[qi][e] += __shfl_xor_sync(0xffffffffu, acc[qi][e], o);
        }
    }
    if (rl != 0) return;
#pragma unroll
    for (int qi = 0; qi < NQ; qi++) {
        if ((uint32_t)qi >= rep) continue;
        const uint32_t h = g * rep + qi;
        const size_t ob = ((size_t)tm.row * P.n_heads + h) * VD;
        const float inv = 1.0f / l[qi];
#pragma unroll
        for (int e = 0; e < EV; e++) {
            const uint32_t d = sub * EV + e;
            float val = acc[qi][e] * inv;
            if (P.gate) val *= 1.0f / (1.0f + ex2(-act_load(P.gate, P.act_dt, ob + d) * 1.4426950408889634f));
            out_store<VD>(P, tm.row, h * VD + d, val);
        }
    }
}

}  // namespace nda
