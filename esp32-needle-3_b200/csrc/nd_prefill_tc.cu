// nd_prefill_tc.cu - causal prefill attention on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA) for 16-bit caches with head dim 64.
//
// Reference semantics: N successive decode steps of the host engine
// (esp32/main/main.c:233-234; per step nd_model.c:2419-2483), i.e. query
// token t at position p = pos0 + t attends to cache positions [0, p] of its
// sequence once every token of the call has been appended (the caller runs K1
// first and guarantees the call does not wrap the ring, so slot == position).
//
// One CTA = one work item = 128 consecutive query tokens of one sequence for
// one query head h (KV head g = h / rep), walking 64-key tiles. 6 warps:
//   warps 0-3  one thread per query row (= TMEM lane): RoPE(+norm) of the Q
//              row, per-row online softmax on S read from TMEM, P written back
//              over S, lazy O rescaling (only when a row max grows by more than
//              2^8), epilogue
//   warp 4     TMA producer: Q tile once, then K/V tiles through a 4-stage ring
//              (contiguous cache rows, or page by page through the block table)
//   warp 5     TMEM allocator + single-thread MMA issuer, an event loop that
//              issues each PV as soon as its P is written and each S as soon
//              as its K tile has landed and its buffer is free:
//                S_j = Q K_j^T  (M=128, N=64, K=64; A = Q from TMEM, B = K smem)
//                O  += P_j V_j  (M=128, N=64, K=64; A = P from TMEM, B = V smem,
//                                MN-major)
// TMEM columns (256 per CTA, 2 CTAs per SM): the S/P double buffer [0,128),
// O [128,192), Q_hi [192,224), Q_lo [224,256). The two CTAs of an SM overlap
// one CTA's softmax with the other's MMAs.
//
// Precision: bf16 rounds a value by up to 2^-9, which rows attending to few
// keys (P) or normed rows with larger |q||k| (Q) turn into output errors above
// 1e-3 (measured ~1.5e-3 and ~2e-3). So with bf16 both operands the kernel
// makes itself carry ~16 mantissa bits as a hi/lo pair: the rotated Q
// (S = Q_hi K^T + Q_lo K^T)
// and P (P_hi/P_lo overwrite the S columns they came from, per 32-key chunk 16
// columns of P_hi then 16 of P_lo; O += P_hi V + P_lo V). K and V are the
// cache's own values, exact already. f16 (11-bit mantissa, errors ~2e-4 and
// ~5e-4) needs no split: one MMA per k-step, P as single f16 pairs. S_{j+NB}
// reuses S_j's columns, so it waits for PV_j.
//
// Every mbarrier wait is bounded (~2 s of SM clock); on expiry the CTA raises
// the error word, drains what it issued (bounded), frees TMEM and returns.
// Every TMA box is loaded by the CTA that reads it.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "nd_async.cuh"
#include "nd_internal.h"
#include "nd_tc.cuh"

namespace nda {
namespace {

constexpr int BM = 128;          // query rows per CTA (TMEM lanes)
constexpr int BN = 64;           // keys per KV tile
constexpr int HD = 64;           // head dim (one 128-byte swizzle row of 16-bit values)
constexpr int NB = 2;            // S/P buffers in TMEM
constexpr int STAGES = 4;        // K/V ring
constexpr uint32_t Q_BYTES = BM * HD * 2;    // 16 KB
constexpr uint32_t KV_BYTES = BN * HD * 2;   // 8 KB per K or V tile
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t COL_S = 0, COL_O = 128, COL_QHI = 192, COL_QLO = 224;

// Dynamic shared memory: Q landing tile, K and V stage rings (1024-byte
// aligned tiles for the 128-byte swizzle), a 32 KB block, then the barrier
// block. The 32 KB block first holds the tile's 128 RoPE table rows (256 B
// each, 16-byte chunks XOR-swizzled by row so per-row reads are conflict-free),
// then the gate tile (TMA) and the output tile for the TMA store (128 rows of
// 128 B, 128-byte swizzle; f32 output: two such boxes).
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = OFF_Q + Q_BYTES;
constexpr uint32_t OFF_V = OFF_K + STAGES * KV_BYTES;
constexpr uint32_t OFF_X = OFF_V + STAGES * KV_BYTES;
constexpr uint32_t X_BYTES = BM * 256;       // 32 KB
constexpr uint32_t OFF_BAR = OFF_X + X_BYTES;

// Per S/P buffer b (tiles j with j % NB == b, phase j / NB): s_full (S
// landed), p_full (P written), pv_done (PV read P and wrote O). Every wait
// below is for the next phase to complete or the one just completed, never
// further away, which is what makes the parity test exact.
struct Bars {
    uint64_t q_full, cs_full, q_ready, stage_full, x_free, drain;
    uint64_t s_full[NB], p_full[NB], pv_done[NB];
    uint64_t kv_full[STAGES], kv_empty[STAGES];
    uint32_t tmem_base;
    int abort_flag;
};
constexpr uint32_t SMEM_BYTES = OFF_BAR + sizeof(Bars);

// P = 2^(S*c - m) for 32 keys of a row, written over their S columns: with
// PSPLIT as hi/lo bf16 pairs (16 columns of hi, then 16 of lo), else as single
// f16 pairs (16 columns). The row sum goes into l2.
template <bool PSPLIT>
__device__ __forceinline__ void write_p_chunk(const uint32_t (&sv)[32], uint32_t taddr, float c, float m, float2 &l2) {
    const float2 c2v = make_float2(c, c), nm2 = make_float2(-m, -m), neg1 = make_float2(-1.0f, -1.0f);
    float2 acc[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
    uint32_t pk[32];
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
        const float2 sp = make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1]));
        const float2 t = __ffma2_rn(sp, c2v, nm2);
        const float2 pp = make_float2(ex2(t.x), ex2(t.y));
        acc[(e >> 1) & 1] = __fadd2_rn(acc[(e >> 1) & 1], pp);
        if constexpr (PSPLIT) {
            // hi = the upper halves (truncated bf16), lo = RN(p - hi): p - hi is
            // exact in fp32, so hi + lo keeps ~16 bits of p.
            const uint32_t u0 = __float_as_uint(pp.x), u1 = __float_as_uint(pp.y);
            pk[e / 2] = __byte_perm(u0, u1, 0x7632);
            const float2 hf = make_float2(__uint_as_float(u0 & 0xffff0000u), __uint_as_float(u1 & 0xffff0000u));
            const float2 lf = __ffma2_rn(hf, neg1, pp);
            pk[16 + e / 2] = pack2<true>(lf.x, lf.y);
        } else {
            pk[e / 2] = pack2<false>(pp.x, pp.y);
        }
    }
    if constexpr (PSPLIT) tmem_st32(taddr, pk);
    else tmem_st16(taddr, pk);
    l2 = __fadd2_rn(l2, __fadd2_rn(acc[0], acc[1]));
}

// BF16 = 16-bit type of the cache and activations. PVF16 (bf16 only): P and
// V in f16 for PV, V tiles converted in shared memory by the softmax warps
// (exact while the layer's V holds no value of |x| >= 2^16, Inf or NaN);
// otherwise P goes as a bf16 hi/lo pair. Both bf16 variants are launched one
// after the other; each exits at once unless the layer's flag selects it.
template <bool BF16, bool PVF16>
__global__ void __launch_bounds__(192, 2)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap omap,
                      const __grid_constant__ CUtensorMap csmap, const PrefillTcParams P) {
    constexpr bool PSPLIT = BF16 && !PVF16;   // P as a bf16 hi/lo pair (two PV MMAs per k-step)
    if constexpr (BF16) {
        const bool big = P.vbig == nullptr || *reinterpret_cast<const volatile int *>(P.vbig) != 0;
        if (big == PVF16) return;   // the other variant serves this call
    }
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (su32(smem_raw) & 1023u) {          // the swizzled tiles need 1024-byte alignment
        if (tid == 0) *reinterpret_cast<volatile int *>(P.err) = 4;
        return;
    }
    uint8_t *sq = smem_raw + OFF_Q;
    Bars &B = *reinterpret_cast<Bars *>(smem_raw + OFF_BAR);
    volatile int *abort_flag = &B.abort_flag;
    // This CTA's items: blockIdx.x, + gridDim.x, ... of the longest-first list.
    const uint32_t n_items = blockIdx.x < P.n_work ? (P.n_work - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    auto item = [&](uint32_t k) { return P.work[blockIdx.x + k * gridDim.x]; };
    auto tiles_of = [](const PrefillWork &w) { return (w.pos0 + w.t0 + w.rows + BN - 1) / BN; };

    if (tid == 0) {
        mbar_init(&B.q_full, 1);
        mbar_init(&B.cs_full, 1);
        mbar_init(&B.q_ready, BM / 32);       // one arrive per softmax warp
        mbar_init(&B.stage_full, BM / 32);
        mbar_init(&B.x_free, 1);
        mbar_init(&B.drain, 1);
        for (int b = 0; b < NB; b++) {
            mbar_init(&B.s_full[b], 1);
            mbar_init(&B.p_full[b], BM / 32);
            mbar_init(&B.pv_done[b], 1);
        }
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&B.kv_full[s], 1);
            mbar_init(&B.kv_empty[s], 1);
        }
        B.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&B.tmem_base)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tbase = B.tmem_base;

    if (warp == 4) {
        // ---------------- TMA producer: per item its Q tile and RoPE rows, then
        // its K/V tiles through the ring (global tile count gt)
        if (lane == 0) {
            uint32_t gt = 0, issued = 0, qi = 0, ci = 0;
            for (uint32_t k = 0; k < n_items && !*abort_flag; k++) {
                const PrefillWork w = item(k);
                // Q landing tile: free once item k-1's rows are in TMEM.
                if (k > 0 && !mbar_wait(&B.q_ready, (k - 1) & 1, abort_flag)) break;
                mbar_expect_tx(&B.q_full, Q_BYTES);
                tma_load_2d(sq, &qmap, (int)(w.head * HD), (int)(w.tok_base + w.t0), &B.q_full);
                qi++;
                // RoPE rows: the 32 KB block is free once item k-2's output
                // tile has been read out of it (x_free, one phase per item).
                if (k > 1 && !mbar_wait(&B.x_free, (k - 2) & 1, abort_flag)) break;
                mbar_expect_tx(&B.cs_full, X_BYTES);
                tma_load_3d(smem_raw + OFF_X, &csmap, 0, 0, (int)(w.pos0 + w.t0), &B.cs_full);
                ci++;
                const uint32_t nkv = tiles_of(w), g = w.head / P.rep, kv_row0 = w.seq * P.window;
                for (uint32_t j = 0; j < nkv; j++, gt++) {
                    const uint32_t st = gt % STAGES;
                    // Cache row of key j * BN: contiguous, or through the block
                    // table (a 64-key tile lies in one page of >= 64 slots).
                    const uint32_t key = j * BN;
                    const int row = P.btab ? (int)(((uint32_t)P.btab[(size_t)w.seq * P.blocks_per_seq +
                                                                       (key >> P.block_shift)]
                                                    << P.block_shift) |
                                                   (key & ((1u << P.block_shift) - 1u)))
                                           : (int)(kv_row0 + key);
                    if (gt >= STAGES && !mbar_wait(&B.kv_empty[st], ((gt / STAGES) - 1) & 1, abort_flag)) break;
                    mbar_expect_tx(&B.kv_full[st], 2 * KV_BYTES);
                    tma_load_2d(smem_raw + OFF_K + st * KV_BYTES, &kmap, (int)(g * HD), row, &B.kv_full[st]);
                    tma_load_2d(smem_raw + OFF_V + st * KV_BYTES, &vmap, (int)(g * HD), row, &B.kv_full[st]);
                    issued = gt + 1;
                }
            }
            if (*abort_flag) {
                // Let the copies this thread issued land before the CTA goes away.
                if (qi) mbar_drain(&B.q_full, (qi - 1) & 1);
                if (ci) mbar_drain(&B.cs_full, (ci - 1) & 1);
                if (issued) mbar_drain(&B.kv_full[(issued - 1) % STAGES], ((issued - 1) / STAGES) & 1);
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer: per item, S one tile ahead of PV
        if (lane == 0) {
            constexpr uint32_t fmt = BF16 ? 1u : 0u;
            constexpr uint32_t id_s = idesc_f16(fmt, BM, BN, 0);
            constexpr uint32_t id_o = idesc_f16(PSPLIT ? 1u : 0u, BM, HD, 1);   // P and V: bf16 pair or f16
            bool ok = true;
            uint32_t issued = 0, gs = 0, gp = 0;     // next S / next PV to issue (global tiles)
            for (uint32_t k = 0; ok && k < n_items; k++) {
                const uint32_t g0 = gp, gend = gp + tiles_of(item(k));
                ok = mbar_wait(&B.q_ready, k & 1, abort_flag);
                // Event loop: issue whatever is ready, PV first (it frees an S
                // buffer), then the next S. A barrier is only tested once the
                // operation it tracks has been issued, so each test is for the
                // next phase or the one just completed (the parity test is exact).
                long long idle_since = clock64();
                while (ok && gp < gend) {
                    bool progressed = false;
                    if (gp < gs && mbar_ready(&B.p_full[gp % NB], (gp / NB) & 1)) {
                        // O += P V (P in S buffer gp % NB, V in stage gp % STAGES).
                        const uint32_t b = gp % NB, st = gp % STAGES;
                        fence_after();
                        const uint32_t v_addr = su32(smem_raw + OFF_V + st * KV_BYTES);
#pragma unroll
                        for (uint32_t kk = 0; kk < BN / 16; kk++) {
                            const uint64_t vd = sdesc(v_addr + kk * 2048, KV_BYTES, 1024);
                            const uint32_t pc = tbase + COL_S + b * BN + 32 * (kk / 2) + 8 * (kk % 2);
                            umma_ts(tbase + COL_O, pc, vd, id_o, (gp > g0 || kk > 0) ? 1u : 0u);
                            if constexpr (PSPLIT) umma_ts(tbase + COL_O, pc + 16, vd, id_o, 1u);
                        }
                        umma_commit(&B.kv_empty[st]);
                        umma_commit(&B.pv_done[b]);
                        gp++;
                        progressed = true;
                    }
                    if (gs < gend && (gs < NB || (gp > gs - NB && mbar_ready(&B.pv_done[gs % NB], (gs / NB - 1) & 1))) &&
                        mbar_ready(&B.kv_full[gs % STAGES], (gs / STAGES) & 1)) {
                        // S = Q K^T into buffer gs % NB (its previous P was read).
                        const uint32_t b = gs % NB, st = gs % STAGES;
                        fence_after();
                        const uint32_t k_addr = su32(smem_raw + OFF_K + st * KV_BYTES);
#pragma unroll
                        for (uint32_t kk = 0; kk < HD / 16; kk++) {
                            const uint64_t kd = sdesc(k_addr + kk * 32, 16, 1024);
                            umma_ts(tbase + COL_S + b * BN, tbase + COL_QHI + kk * 8, kd, id_s, kk > 0);
                            if constexpr (BF16)
                                umma_ts(tbase + COL_S + b * BN, tbase + COL_QLO + kk * 8, kd, id_s, 1u);
                        }
                        umma_commit(&B.s_full[b]);
                        gs++;
                        issued = 1;
                        progressed = true;
                    }
                    if (progressed) {
                        idle_since = clock64();
                    } else if (*abort_flag) {
                        ok = false;
                    } else if (clock64() - idle_since > kTimeoutCycles) {
                        *abort_flag = 1;
                        ok = false;
                    }
                }
            }
            if (*abort_flag && issued) {
                umma_commit(&B.drain);
                mbar_drain(&B.drain, 0);
            }
        }
    } else {
        // ---------------- softmax / correction / epilogue: thread = query row
        const uint32_t r = tid;
        const uint32_t lane_addr = tbase + ((uint32_t)(warp * 32) << 16);
        // Softmax scale in log2 units; with f16 queries, times the power of two
        // this row's Q was scaled down by (set per item in setup).
        float c = P.scale_log2;
        bool ok = true, store_pending = false;
        uint32_t n_stores = 0;

        // Set-up of item k: RoPE (after the optional per-head norm) of this
        // row, split hi/lo into TMEM as the A operand of S = Q K^T. The Q TMEM
        // columns are free: the previous item's last S has completed.
        auto setup = [&](uint32_t k) {
            const PrefillWork w = item(k);
            ok = ok && __all_sync(0xffffffffu, mbar_wait(&B.q_full, k & 1, abort_flag));
            ok = ok && __all_sync(0xffffffffu, mbar_wait(&B.cs_full, k & 1, abort_flag));
            if (!ok) return;
            float x[HD];
#pragma unroll
            for (int cq = 0; cq < 8; cq++) {
                const uint4 u = *reinterpret_cast<const uint4 *>(sq + swz(r, cq));
                const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 f = unpack2<BF16>(uu[e]);
                    x[cq * 8 + 2 * e] = f.x;
                    x[cq * 8 + 2 * e + 1] = f.y;
                }
            }
            // The queries only need the output tolerance (the bit-exact
            // statement order matters for the cached K, not here): the norm is
            // applied once up front, the rotation as packed FMAs, and the
            // per-element branches stay outside the loops.
            if (P.qnorm) {
                float ss = 0.0f;
#pragma unroll
                for (int i = 0; i < HD; i++) ss = fmaf(x[i], x[i], ss);
                const float inv = rsqrtf(ss * (1.0f / HD) + 1e-6f);
#pragma unroll
                for (int i = 0; i < HD; i++) x[i] *= (1.0f + P.qnorm[i]) * inv;
            }
#pragma unroll
            for (int i = 0; i < HD / 2; i += 2) {
                const float4 t4 = *reinterpret_cast<const float4 *>(smem_raw + OFF_X + cs_off(r, i >> 1));
                // pairs i and i+1: (a, b) -> (a c - b s, b c + a s)
                const float2 a2 = make_float2(x[i], x[i + 1]), b2 = make_float2(x[i + HD / 2], x[i + 1 + HD / 2]);
                const float2 c2 = make_float2(t4.x, t4.z), s2 = make_float2(t4.y, t4.w);
                const float2 ra = __ffma2_rn(a2, c2, __fmul2_rn(make_float2(-b2.x, -b2.y), s2));
                const float2 rb = __ffma2_rn(b2, c2, __fmul2_rn(a2, s2));
                x[i] = ra.x, x[i + 1] = ra.y, x[i + HD / 2] = rb.x, x[i + 1 + HD / 2] = rb.y;
            }
            uint32_t hi[32];
            if constexpr (BF16) {
                uint32_t lo[32];
#pragma unroll
                for (int e = 0; e < 32; e++) split2<true>(x[2 * e], x[2 * e + 1], hi[e], lo[e]);
                tmem_st32(lane_addr + COL_QHI, hi);
                tmem_st32(lane_addr + COL_QLO, lo);
            } else {
                // f16 queries: the row scaled by 2^-e so that its largest |q|
                // stays below 2^15 (RoPE can push an f16 input past 65504);
                // exact, a power of two. S comes out 2^-e too small and the
                // row's scale c takes 2^e.
                float amax = 0.0f;
#pragma unroll
                for (int i = 0; i < HD; i++) amax = fmaxf(amax, fabsf(x[i]));
                const int e = max(0, (int)((__float_as_uint(amax) >> 23) & 0xffu) - 127 - 14);
                const float down = __uint_as_float((uint32_t)(127 - min(e, 126)) << 23);
#pragma unroll
                for (int i = 0; i < 32; i++) hi[i] = pack2<false>(x[2 * i] * down, x[2 * i + 1] * down);
                c = P.scale_log2 * __uint_as_float((uint32_t)(127 + min(e, 127)) << 23);
                tmem_st32(lane_addr + COL_QHI, hi);
            }
            tmem_wait_st();
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.q_ready);
        };
        // The previous output tile has been read out of the 32 KB block.
        auto release_x = [&]() {
            if (tid == 0 && store_pending) {
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                mbar_arrive(&B.x_free);
                store_pending = false;
            }
        };

        if (n_items) setup(0);
        uint32_t gt = 0;
        for (uint32_t k = 0; ok && k < n_items; k++) {
            const PrefillWork w = item(k);
            const uint32_t nkv = tiles_of(w), g0 = gt;
            const uint32_t qpos = w.pos0 + w.t0 + r;                  // this row's position
            const bool row_valid = r < w.rows;
            float m = -INFINITY;
            float2 l2 = make_float2(0.0f, 0.0f);   // row sum of P, two partial sums
            for (uint32_t j = 0; j < nkv; j++, gt++) {
                const uint32_t b = gt % NB, sbuf = lane_addr + COL_S + b * BN;
                if (!__all_sync(0xffffffffu, mbar_wait(&B.s_full[b], (gt / NB) & 1, abort_flag))) {
                    ok = false;
                    break;
                }
                fence_after();
                const int lim = (int)qpos - (int)(j * BN);   // keys [0, lim] of this tile are visible
                const bool masked = !__all_sync(0xffffffffu, lim >= BN - 1);   // tile crosses the warp's diagonal
                // Pass 1: the tile's row max (8 independent chains per 32 columns),
                // both 32-column loads in flight before one wait.
                float mx[8];
#pragma unroll
                for (int kq = 0; kq < 8; kq++) mx[kq] = -INFINITY;
                uint32_t sv2[BN / 32][32];
#pragma unroll
                for (int c2 = 0; c2 < BN / 32; c2++) tmem_ld32_async(sbuf + 32 * c2, sv2[c2]);
                tmem_wait_ld();
#pragma unroll
                for (int c2 = 0; c2 < BN / 32; c2++) {
                    uint32_t(&sv)[32] = sv2[c2];
                    if (masked) {
#pragma unroll
                        for (int e = 0; e < 32; e++)
                            if (c2 * 32 + e > lim) sv[e] = 0xff800000u;
                    }
#pragma unroll
                    for (int e = 0; e < 32; e += 2)
                        mx[(e >> 1) & 7] = fmax3(mx[(e >> 1) & 7], __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]));
                }
#pragma unroll
                for (int w2 = 4; w2 > 0; w2 >>= 1)
#pragma unroll
                    for (int kq = 0; kq < w2; kq++) mx[kq] = fmaxf(mx[kq], mx[kq + w2]);
                const float tmax = mx[0] * c;
                // Lazy rescale: keep the running max unless a row's max grew by
                // more than 2^8; then O and l move to the new max (the previous
                // PV is done: this S was issued after it).
                const bool grow = j == 0 || tmax > m + 8.0f;
                if (j > 0 && __any_sync(0xffffffffu, grow)) {
                    if (!__all_sync(0xffffffffu,
                                    mbar_wait(&B.pv_done[(gt - 1) % NB], ((gt - 1) / NB) & 1, abort_flag))) {
                        ok = false;
                        break;
                    }
                    fence_after();
                    const float alpha = grow ? ex2(m - tmax) : 1.0f;
                    l2 = __fmul2_rn(l2, make_float2(alpha, alpha));
                    // 16 columns at a time: this tile's 64 S values stay live.
                    uint32_t ov[16];
#pragma unroll
                    for (int h2 = 0; h2 < HD / 16; h2++) {
                        tmem_ld16(lane_addr + COL_O + h2 * 16, ov);
#pragma unroll
                        for (int e = 0; e < 16; e++) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
                        tmem_st16(lane_addr + COL_O + h2 * 16, ov);
                    }
                }
                if (grow) m = tmax;
                // Pass 2: P = 2^(S*c - m) over the S columns, from the values
                // pass 1 loaded (masked already).
#pragma unroll
                for (int c2 = 0; c2 < BN / 32; c2++) write_p_chunk<PSPLIT>(sv2[c2], sbuf + 32 * c2, c, m, l2);
                if constexpr (BF16 && PVF16) {
                    // V tile of this stage to f16 in place (exact: the layer's
                    // V holds no value f16 cannot represent), a quarter per warp.
                    uint4 *vt = reinterpret_cast<uint4 *>(smem_raw + OFF_V + (gt % STAGES) * KV_BYTES);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        uint4 u = vt[r + i * BM];
                        uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            wv[e] = pack2<false>(__uint_as_float(wv[e] << 16), __uint_as_float(wv[e] & 0xffff0000u));
                        vt[r + i * BM] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> MMA reads
                }
                tmem_wait_st();
                fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&B.p_full[b]);
                if (j == 0) release_x();
            }
            if (!ok) break;
            // The next item's queries go into TMEM now (its first S can run
            // under this item's epilogue).
            if (k + 1 < n_items) setup(k + 1);
            // O is final once the last PV of every buffer is done.
            for (uint32_t t = gt - g0 > NB ? gt - NB : g0; ok && t < gt; t++)
                if (!__all_sync(0xffffffffu, mbar_wait(&B.pv_done[t % NB], (t / NB) & 1, abort_flag))) ok = false;
            if (!ok) break;
            fence_after();
            const float inv_l = 1.0f / (l2.x + l2.y);
            if (w.rows == BM) {
                // Whole tile: this row's output into the 32 KB block (128-byte
                // swizzle, the layout of the output map), then one TMA store.
                // Both halves of the row first, then straight-line packing and
                // stores with the output type and the gate decided outside the
                // loops (the per-element form of this epilogue cost ~5x more).
                uint32_t oa[32], ob[32];
                tmem_ld32_async(lane_addr + COL_O, oa);
                tmem_ld32_async(lane_addr + COL_O + 32, ob);
                tmem_wait_ld();
                float va[32], vb[32];
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    va[e] = __uint_as_float(oa[e]) * inv_l;
                    vb[e] = __uint_as_float(ob[e]) * inv_l;
                }
                if (P.gate) {
                    const size_t obase = ((size_t)(w.tok_base + w.t0 + r) * P.n_heads + w.head) * HD;
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        va[e] *= 1.0f / (1.0f + ex2(-act_load(P.gate, P.act_dt, obase + e) * 1.4426950408889634f));
                        vb[e] *= 1.0f / (1.0f + ex2(-act_load(P.gate, P.act_dt, obase + 32 + e) * 1.4426950408889634f));
                    }
                }
                // The block still holds item k+1's RoPE rows, which every
                // softmax warp reads in its set-up of item k+1; this row's
                // output lands on another warp's rows (row r's 128 bytes are
                // RoPE row r/2's, the f32 second box rows 64 + r/2). Write only
                // once all four warps have finished that set-up (q_ready's
                // phase for item k+1 completes with their four arrivals).
                if (k + 1 < n_items &&
                    !__all_sync(0xffffffffu, mbar_wait(&B.q_ready, (k + 1) & 1, abort_flag))) {
                    ok = false;
                    break;
                }
                if (P.out_dt == DT_F32) {
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        *reinterpret_cast<float4 *>(smem_raw + OFF_X + swz(r, e)) =
                            make_float4(va[4 * e], va[4 * e + 1], va[4 * e + 2], va[4 * e + 3]);
                        *reinterpret_cast<float4 *>(smem_raw + OFF_X + Q_BYTES + swz(r, e)) =
                            make_float4(vb[4 * e], vb[4 * e + 1], vb[4 * e + 2], vb[4 * e + 3]);
                    }
                } else if (P.out_dt == DT_BF16) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        *reinterpret_cast<uint4 *>(smem_raw + OFF_X + swz(r, e)) =
                            make_uint4(pack2<true>(va[8 * e], va[8 * e + 1]), pack2<true>(va[8 * e + 2], va[8 * e + 3]),
                                       pack2<true>(va[8 * e + 4], va[8 * e + 5]), pack2<true>(va[8 * e + 6], va[8 * e + 7]));
                        *reinterpret_cast<uint4 *>(smem_raw + OFF_X + swz(r, 4 + e)) =
                            make_uint4(pack2<true>(vb[8 * e], vb[8 * e + 1]), pack2<true>(vb[8 * e + 2], vb[8 * e + 3]),
                                       pack2<true>(vb[8 * e + 4], vb[8 * e + 5]), pack2<true>(vb[8 * e + 6], vb[8 * e + 7]));
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        *reinterpret_cast<uint4 *>(smem_raw + OFF_X + swz(r, e)) =
                            make_uint4(pack2<false>(va[8 * e], va[8 * e + 1]), pack2<false>(va[8 * e + 2], va[8 * e + 3]),
                                       pack2<false>(va[8 * e + 4], va[8 * e + 5]), pack2<false>(va[8 * e + 6], va[8 * e + 7]));
                        *reinterpret_cast<uint4 *>(smem_raw + OFF_X + swz(r, 4 + e)) =
                            make_uint4(pack2<false>(vb[8 * e], vb[8 * e + 1]), pack2<false>(vb[8 * e + 2], vb[8 * e + 3]),
                                       pack2<false>(vb[8 * e + 4], vb[8 * e + 5]), pack2<false>(vb[8 * e + 6], vb[8 * e + 7]));
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> TMA reads
                fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&B.stage_full);
                if (tid == 0) {
                    if (!mbar_wait(&B.stage_full, n_stores & 1, abort_flag)) {
                        ok = false;
                    } else {
                        const int y = (int)(w.tok_base + w.t0);
                        tma_store_2d(&omap, smem_raw + OFF_X, (int)(w.head * HD), y);
                        if (P.out_dt == DT_F32)
                            tma_store_2d(&omap, smem_raw + OFF_X + Q_BYTES, (int)(w.head * HD + 32), y);
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                        store_pending = true;
                    }
                }
                n_stores++;
            } else {
                // Partial tile (the end of a sequence): direct row stores, with
                // the gate and the output type decided outside the loops.
                uint32_t oa[32], ob[32];
                tmem_ld32_async(lane_addr + COL_O, oa);
                tmem_ld32_async(lane_addr + COL_O + 32, ob);
                tmem_wait_ld();
                if (row_valid) {
                    const size_t obase = ((size_t)(w.tok_base + w.t0 + r) * P.n_heads + w.head) * HD;
                    float val[HD];
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        val[e] = __uint_as_float(oa[e]) * inv_l;
                        val[32 + e] = __uint_as_float(ob[e]) * inv_l;
                    }
                    if (P.gate) {
#pragma unroll
                        for (int e = 0; e < HD; e++)
                            val[e] *= 1.0f / (1.0f + ex2(-act_load(P.gate, P.act_dt, obase + e) * 1.4426950408889634f));
                    }
                    if (P.out_dt == DT_F32) {
                        float4 *o4 = reinterpret_cast<float4 *>(static_cast<float *>(P.out) + obase);
#pragma unroll
                        for (int e = 0; e < HD / 4; e++)
                            o4[e] = make_float4(val[4 * e], val[4 * e + 1], val[4 * e + 2], val[4 * e + 3]);
                    } else if (P.out_dt == DT_BF16) {
                        uint4 *o4 = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(P.out) + obase);
#pragma unroll
                        for (int e = 0; e < HD / 8; e++)
                            o4[e] = make_uint4(pack2<true>(val[8 * e], val[8 * e + 1]),
                                               pack2<true>(val[8 * e + 2], val[8 * e + 3]),
                                               pack2<true>(val[8 * e + 4], val[8 * e + 5]),
                                               pack2<true>(val[8 * e + 6], val[8 * e + 7]));
                    } else {
                        uint4 *o4 = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(P.out) + obase);
#pragma unroll
                        for (int e = 0; e < HD / 8; e++)
                            o4[e] = make_uint4(pack2<false>(val[8 * e], val[8 * e + 1]),
                                               pack2<false>(val[8 * e + 2], val[8 * e + 3]),
                                               pack2<false>(val[8 * e + 4], val[8 * e + 5]),
                                               pack2<false>(val[8 * e + 6], val[8 * e + 7]));
                    }
                }
                // The 32 KB block was not used: released at once.
                fence_before();
                __syncwarp();
                if (tid == 0) mbar_arrive(&B.x_free);
            }
            // O is read: the next item's first PV may overwrite it (its P is
            // only written after this point).
            tmem_wait_ld();
        }
        if (tid == 0 && store_pending) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }

    fence_before();
    __syncthreads();
    if (tid == 0 && B.abort_flag) *reinterpret_cast<volatile int *>(P.err) = 3;
    if (warp == 5) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TMEM_COLS));
    }
}

}  // namespace

size_t prefill_tc_smem_bytes() { return SMEM_BYTES; }

template <bool BF16, bool PVF16>
cudaError_t prefill_tc_launch_t(const CUtensorMap &q, const CUtensorMap &k, const CUtensorMap &v,
                                const CUtensorMap &o, const CUtensorMap &cs, const PrefillTcParams &P, uint32_t grid,
                                cudaStream_t s) {
    const size_t smem = prefill_tc_smem_bytes();
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel<BF16, PVF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    prefill_tc_kernel<BF16, PVF16><<<grid, 192, smem, s>>>(q, k, v, o, cs, P);
    return cudaGetLastError();
}

cudaError_t prefill_tc_launch(bool bf16, const void *qmap, const void *kmap, const void *vmap, const void *omap,
                              const void *csmap, const PrefillTcParams &P, uint32_t grid, cudaStream_t s) {
    const CUtensorMap &q = *static_cast<const CUtensorMap *>(qmap);
    const CUtensorMap &k = *static_cast<const CUtensorMap *>(kmap);
    const CUtensorMap &v = *static_cast<const CUtensorMap *>(vmap);
    const CUtensorMap &o = *static_cast<const CUtensorMap *>(omap);
    const CUtensorMap &cs = *static_cast<const CUtensorMap *>(csmap);
    if (!bf16) return prefill_tc_launch_t<false, false>(q, k, v, o, cs, P, grid, s);
    // bf16: the f16-PV variant, then the hi/lo variant; the layer's flag on
    // the device makes one of them exit at once.
    cudaError_t e = prefill_tc_launch_t<true, true>(q, k, v, o, cs, P, grid, s);
    if (e != cudaSuccess) return e;
    return prefill_tc_launch_t<true, false>(q, k, v, o, cs, P, grid, s);
}

}  // namespace nda
