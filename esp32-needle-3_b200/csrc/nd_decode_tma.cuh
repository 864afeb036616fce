// nd_decode_tma.cuh - persistent, dynamically balanced split-KV attention with
// the K/V rows staged by TMA.
//
// Same results as attend_kernel (nd_device.cuh) for 16-bit and int8 caches
// whose head dims are equal (64 or 128) and calls in which no position wraps
// the ring (visit index == slot == position).
//
// Work. Item (t, g) = query token t, KV head g; it holds T_t tiles of TR cache
// rows (64; 128 for int8 caches). Items are concatenated token-major into NT
// tiles, cut into units:
// G static units of S tiles (CTA c starts with unit c), then dynamic units of
// CH tiles that CTAs take from a global counter as they run dry, so an SM that
// the memory system serves faster takes more work and all CTAs end together.
// G = the CTAs the GPU holds at once: one wave, persistent. A unit can start
// or end inside an item; an item's pieces (one per unit it overlaps) leave
// partial (m, l, acc) rows, and the last piece to take the item's ticket
// merges them (no CTA ever waits for another). A global-memory round trip
// takes several us while the memory system is saturated, so a CTA takes its
// tickets only when it runs out of work: one fence, then one ticket per lane.
//
// Roles (warps). 0..3 consume tiles (the lane mapping and online softmax of
// attend_kernel, rows read from shared memory); 4 = producer: takes units,
// publishes a descriptor per segment (maximal run of one item inside a unit)
// into a SQ-deep slot ring and issues the TMA boxes (2D maps over
// [rows][n_kv * hd], box hd x TR, each CTA loading its own) into a STAGES-deep ring;
// 5 = prep: query rows of each segment (norm + RoPE) and the fused append of
// the newest row; 6 = finisher: merges the consumers' per-warp results of a
// segment and writes the output, or the item's partial and a note of it in
// shared memory, so the merge does not sit on the consumers' path. Every mbarrier wait is bounded (nd_async.cuh); on a timeout
// each role stops (no named barriers, so none can be left waiting).
//
// Paged caches work when a page holds a whole number of tiles: tiles start on
// multiples of TR rows of an item, so every box lies in one page.
//
// Launch overlap (programmatic dependent launch): the kernel may start while
// the previous kernel on the stream still runs. The prep and finisher warps
// wait for it (griddepcontrol.wait) before touching the caller's tensors; the
// producer streams K/V before that only when P.early_kv says the previous
// kernel cannot be writing this layer's cache. Once its prep warp has waited,
// each CTA lets the next launch start (griddepcontrol.launch_dependents), so at
// most two launches overlap: they use alternate halves of the counters and of
// the partial scratch. The tail of one launch (last pieces, merges) thereby
// runs under the start of the next.
#pragma once
#include "nd_async.cuh"
#include "nd_device.cuh"

namespace nda {

#ifndef ND_LEAN_STAGES64
#define ND_LEAN_STAGES64 4
#endif
// Units a producer takes ahead of the one it streams (P.lean_ahead, 1..4): the
// queue atomic has the loaded memory latency, longer than a short unit takes.
constexpr int kLeanAheadMax = 4;

template <int HD, typename KVT, int NQ> struct LeanCfg {
    static constexpr bool I8 = KvT<KVT>::dt == DT_I8;
    static constexpr int NW = 4;                                     // consumer warps
    static constexpr int TR = lean_rows(I8);                         // rows per tile
    // Tile ring depth (int8: 128-row tiles).
    static constexpr int STAGES = I8 ? (HD == 64 ? 3 : 2) : HD == 64 ? ND_LEAN_STAGES64 : (NQ >= 4 ? 2 : 3);
    static constexpr int SQ = NQ * HD >= 256 ? 2 : 4;                // segment slot ring depth
    // CTAs per SM the register budget is sized for: one query row at hd 64 fits
    // three (the shared-memory limit too) in 96 registers without spills.
    static constexpr int MINB = NQ == 1 && HD == 64 ? 3 : 1;
    static constexpr uint32_t TILE = TR * HD * sizeof(KVT);
    // An item's last tile loads only the 16-row sub-boxes that hold its rows.
    static constexpr int SUBR = 16;
    static constexpr uint32_t SUB = SUBR * HD * sizeof(KVT);
    // int8: per stage the K and V scales of the tile's rows for four KV heads
    // (a {4, TR} f32 box: TMA moves at least 16 bytes per row).
    static constexpr uint32_t SC = I8 ? TR * 16 : 0;
    static constexpr uint32_t OFF_V = STAGES * TILE;
    static constexpr uint32_t OFF_KS = 2 * STAGES * TILE;                       // [STAGES][TR][4] f32
    static constexpr uint32_t OFF_VS = OFF_KS + STAGES * SC;
    static constexpr uint32_t OFF_Q = OFF_KS + 2 * STAGES * SC;                 // [SQ][NQ][HD] f32
    static constexpr uint32_t OFF_MO = OFF_Q + SQ * NQ * HD * 4;                // [SQ][NW][NQ][HD] f32
    static constexpr uint32_t OFF_ML = OFF_MO + SQ * NW * NQ * HD * 4;          // [SQ][NW][NQ][2] f32
    static constexpr uint32_t SMEM = OFF_ML + SQ * NW * NQ * 2 * 4;
};

// int8 rows: q.k on the integer dot-product path. A segment's query row q
// (already scaled by scale * log2 e) is held as q = c * (l2 * 2^16 + l1 * 2^8 + l0),
// a 23-bit fixed-point integer in three byte limbs (l2 signed, l1 and l0
// unsigned) with c = 2^-sh a power of two picked from the row's largest |q|
// (|q / c| < 2^22), so q.k over four cache bytes is one dp4a per limb, exact in
// int32, and the three sums meet in f32. Quantising q costs at most 2^-23 of
// the row's largest element: the size of the rounding the reference's own
// float dot product makes (qk_dot8 in attn_heads, nd_model.c:2188-2214). A
// non-finite query element makes c NaN, so the row's scores are NaN as with
// float arithmetic.
template <int NQ, int EK, int LPR>
__device__ __forceinline__ void q_limbs(const float (&qr)[NQ][EK], uint32_t (&ql)[NQ][3][EK / 4],
                                        float (&cq)[NQ][3]) {
#pragma unroll
    for (int qi = 0; qi < NQ; qi++) {
        float mx = 0.0f, z = 0.0f;
#pragma unroll
        for (int e = 0; e < EK; e++) {
            mx = fmaxf(mx, fabsf(qr[qi][e]));
            z += qr[qi][e] * 0.0f;   // NaN when any element is Inf or NaN
        }
#pragma unroll
        for (int o = 1; o < LPR; o <<= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            z += __shfl_xor_sync(0xffffffffu, z, o);
        }
        // mx < 2^ex; scale by 2^sh, sh = 22 - ex, kept inside the normal range.
        const int ex = (int)((__float_as_uint(mx) >> 23) & 0xffu) - 126;
        const int sh = min(126, max(-126, 22 - ex));
        const float up = __uint_as_float((uint32_t)(127 + sh) << 23);
        const float c = __uint_as_float((uint32_t)(127 - sh) << 23) + z;
        cq[qi][0] = c;
        cq[qi][1] = c * 256.0f;
        cq[qi][2] = c * 65536.0f;
#pragma unroll
        for (int w = 0; w < EK / 4; w++) {
            uint32_t b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int x = z == 0.0f ? __float2int_rn(qr[qi][4 * w + j] * up) : 0;
                b0 |= ((uint32_t)x & 0xffu) << (8 * j);
                b1 |= ((uint32_t)(x >> 8) & 0xffu) << (8 * j);
                b2 |= ((uint32_t)(x >> 16) & 0xffu) << (8 * j);
            }
            ql[qi][0][w] = b0;
            ql[qi][1][w] = b1;
            ql[qi][2][w] = b2;
        }
    }
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// This lane's partial q.k of each row group from its K words (EK int8 values).
template <int NQ, int EK, int UU>
__device__ __forceinline__ void qk_i8dp(const uint32_t (&ql)[NQ][3][EK / 4], const float (&cq)[NQ][3],
                                        const uint32_t (&kw)[UU][EK / 4], float (&s)[UU][NQ]) {
#pragma unroll
    for (int u = 0; u < UU; u++)
#pragma unroll
        for (int qi = 0; qi < NQ; qi++) {
            int a2 = 0, a1 = 0, a0 = 0;
#pragma unroll
            for (int w = 0; w < EK / 4; w++) {
                a2 = dp4a_ss(ql[qi][2][w], kw[u][w], a2);
                a1 = dp4a_us(ql[qi][1][w], kw[u][w], a1);
                a0 = dp4a_us(ql[qi][0][w], kw[u][w], a0);
            }
            s[u][qi] = fmaf((float)a2, cq[qi][2], fmaf((float)a1, cq[qi][1], (float)a0 * cq[qi][0]));
        }
}

template <int HD, typename KVT, int NQ>
constexpr uint32_t attend_lean_smem_bytes() {
    return LeanCfg<HD, KVT, NQ>::SMEM;
}

// Unit geometry: G static units of S tiles, then dynamic units of CH tiles.
struct LeanUnits {
    uint32_t G, S, CH, NT, NU;
    __device__ __forceinline__ uint32_t start(uint32_t u) const {
        const uint64_t x = u < G ? (uint64_t)u * S : (uint64_t)G * S + (uint64_t)(u - G) * CH;
        return x < NT ? (uint32_t)x : NT;
    }
    __device__ __forceinline__ uint32_t unit_of(uint32_t x) const {
        const uint32_t ns = G * S;
        return x < ns ? x / S : G + (x - ns) / CH;
    }
};

// Position in the item list: token t (q row t), KV head g, tile kt of the
// item; T tiles per item of the token, base = first tile of the token, and
// the token's sequence and position. Per token {base, T, seq, pos} (uint4)
// comes from a table the host builds: for calls of at most kLeanParamTok
// tokens it is a kernel parameter (LeanTok) and a unit's walk state is found by
// binary search over it; for larger calls the host uploads it (P.split_cu)
// with, per unit, the walk state at its first tile (P.cta_tok, two uint4): one
// global load starts a unit, where a chain of dependent lookups would cost
// several round trips.
struct LeanWalk {
    uint32_t t, g, kt, T, base, seq, pos;
    const uint4 *tab;
    __device__ __forceinline__ void load_token() {
        const uint4 v = tab[t];
        base = v.x, T = v.y, seq = v.z, pos = v.w;
    }
    __device__ __forceinline__ void init(const AttnParams &P, uint32_t u) {
        tab = reinterpret_cast<const uint4 *>(P.split_cu);
        const uint4 a = reinterpret_cast<const uint4 *>(P.cta_tok)[2 * u];
        const uint4 b = reinterpret_cast<const uint4 *>(P.cta_tok)[2 * u + 1];
        t = a.x, g = a.y, kt = a.z, T = a.w, base = b.x, seq = b.y, pos = b.z;
    }
    // Walk state at tile x0 (below the call's total) of a table of ntok
    // tokens: the last token whose first tile is <= x0 (every token holds at
    // least one tile per KV head, so first tiles strictly increase).
    __device__ __forceinline__ void init_at(const uint4 *tab_, uint32_t ntok, uint32_t x0) {
        tab = tab_;
        uint32_t lo = 0, hi = ntok;
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) / 2;
            if (tab[mid].x <= x0) lo = mid;
            else hi = mid;
        }
        t = lo;
        load_token();
        const uint32_t r = x0 - base;
        g = r / T;
        kt = r - g * T;
    }
    __device__ __forceinline__ uint32_t item_start() const { return base + g * T; }
    // Advances past nt tiles of the current item (nt <= T - kt).
    __device__ __forceinline__ void advance(const AttnParams &P, uint32_t nt) {
        kt += nt;
        if (kt < T) return;
        kt = 0;
        if (++g < P.c.n_kv) return;
        g = 0;
        if (++t < P.n_tok) load_token();
    }
};

// Output row qi of the item that starts at tile istart and holds T tiles,
// merged by one warp from the partials of its pieces (slot 2u + (item starts
// inside u)), rescaling the running sums as the max grows. Lane c holds
// output elements c, c + 32, ...; every piece's (m, l) and o are loaded in
// one round of up to eight pieces: one L2 round trip per eight pieces.
template <int HD, int NQ>
__device__ __forceinline__ void lean_merge_row(const AttnParams &P, const LeanUnits &U, uint32_t istart,
                                               uint32_t T, uint32_t g, uint32_t row, int qi, int lane) {
    constexpr int EPL = HD / 32;
    const uint32_t kf = U.unit_of(istart), kl = U.unit_of(istart + T - 1);
    float M = -INFINITY, L = 0.0f, o[EPL];
#pragma unroll
    for (int c = 0; c < EPL; c++) o[c] = 0.0f;
    for (uint32_t u0 = kf; u0 <= kl; u0 += 8) {
        float mp[8], lp[8], op[8][EPL];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            mp[j] = -INFINITY;
            lp[j] = 0.0f;
#pragma unroll
            for (int c = 0; c < EPL; c++) op[j][c] = 0.0f;
            if (u0 + j <= kl) {
                const uint32_t uu = u0 + j, sl = 2 * uu + (istart > U.start(uu) ? 1u : 0u);
                const size_t bq = (size_t)sl * NQ + qi;
                const float2 ml = __ldcg(reinterpret_cast<const float2 *>(P.part_ml) + bq);
                mp[j] = ml.x;
                lp[j] = ml.y;
#pragma unroll
                for (int c = 0; c < EPL; c++) op[j][c] = __ldcg(&P.part_o[bq * HD + lane + 32 * c]);
            }
        }
        float Mn = M;
#pragma unroll
        for (int j = 0; j < 8; j++) Mn = fmaxf(Mn, mp[j]);
        const float sc = ex2(M - Mn);
        L *= sc;
#pragma unroll
        for (int c = 0; c < EPL; c++) o[c] *= sc;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float f = ex2(mp[j] - Mn);
            L += lp[j] * f;
#pragma unroll
            for (int c = 0; c < EPL; c++) o[c] += op[j][c] * f;
        }
        M = Mn;
    }
    const uint32_t col = (g * P.rep + qi) * HD + lane;
    const size_t ob = (size_t)row * P.n_heads * HD + col;
    const float inv = 1.0f / L;
#pragma unroll
    for (int c = 0; c < EPL; c++) {
        float val = o[c] * inv;
        if (P.gate) val *= 1.0f / (1.0f + ex2(-act_load(P.gate, P.act_dt, ob + 32 * c) * 1.4426950408889634f));
        out_store<HD>(P, row, col + 32 * c, val);
    }
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

struct LeanDesc {   // one segment, written by the producer
    uint32_t t, g, kt, nt, T, istart, unit, stop, seq, pos;
};
struct LeanInfo {   // the same segment, completed by the prep warp
    uint32_t row, pos, jend, seq;
    int appender;
};

template <int HD, typename KVT, int NQ>
__global__ void __launch_bounds__(224, (LeanCfg<HD, KVT, NQ>::MINB)) attend_lean_kernel(const __grid_constant__ CUtensorMap kmap,
                                                          const __grid_constant__ CUtensorMap vmap,
                                                          const __grid_constant__ CUtensorMap ksmap,
                                                          const __grid_constant__ CUtensorMap vsmap,
                                                          const __grid_constant__ CUtensorMap ktmap,
                                                          const __grid_constant__ CUtensorMap vtmap,
                                                          const __grid_constant__ LeanTok tk,
                                                          const AttnParams P) {
    using C = LeanCfg<HD, KVT, NQ>;
    using S = AttendShape<HD, HD, KVT, NQ>;
    constexpr int NW = C::NW, TR = C::TR, STAGES = C::STAGES, SQ = C::SQ;
    constexpr int PRODUCER = NW, PREP = NW + 1, FINISH = NW + 2;
    constexpr int LPR = S::LPR, RPW = S::RPW, EK = S::EK, EV = S::EV, WK = S::WK, WV = S::WV, ES = S::ES;
    constexpr int RW = TR / NW;              // rows per warp per tile
    constexpr int UB = RW / RPW < 4 ? RW / RPW : 4;   // row groups per consume call
    constexpr int NCALL = RW / (RPW * UB);   // consume calls per tile
    static_assert(RW % (RPW * UB) == 0, "tile rows split evenly");
    constexpr uint32_t TILE_BYTES = C::TILE;

    extern __shared__ __align__(128) uint8_t smem[];
    float(*sq)[NQ][HD] = reinterpret_cast<float(*)[NQ][HD]>(smem + C::OFF_Q);
    float(*mo)[NW][NQ][HD] = reinterpret_cast<float(*)[NW][NQ][HD]>(smem + C::OFF_MO);
    float(*mml)[NW][NQ][2] = reinterpret_cast<float(*)[NW][NQ][2]>(smem + C::OFF_ML);
    __shared__ LeanDesc desc[SQ];
    __shared__ LeanInfo info[SQ];
    __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES];
    __shared__ __align__(8) uint64_t desc_full[SQ], q_full[SQ], app_full[SQ], mb_full[SQ], slot_free[SQ], settle_bar;
    __shared__ uint32_t pend[32][4];   // split pieces written by the finisher: istart, T, g, out row
    __shared__ uint32_t s_nlast;       // pend[0, s_nlast) = items this CTA completed at its stop
    __shared__ int abort_flag_s;
    volatile int *abort_flag = &abort_flag_s;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t n_kv = P.c.n_kv, W = P.c.window, rep = P.rep;
    const LeanUnits U{P.n_cta, P.lean_s, P.lean_ch, P.n_tiles, P.n_units};
    int *const work_ctr = P.counters + P.work_slot;   // next dynamic unit - G
    int *const done_ctr = work_ctr + 1;               // CTAs finished

    if (tid == 0) {
        for (int s2 = 0; s2 < STAGES; s2++) {
            mbar_init(&full[s2], 1);
            mbar_init(&empty[s2], NW);
        }
        for (int i = 0; i < SQ; i++) {
            mbar_init(&desc_full[i], 1);
            mbar_init(&q_full[i], 1);
            mbar_init(&app_full[i], 1);
            mbar_init(&mb_full[i], NW);
            mbar_init(&slot_free[i], 1);
        }
        mbar_init(&settle_bar, 1);
        abort_flag_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // At its stop every warp helps merge the items this CTA completed (the
    // finisher publishes them through settle_bar): one (item, query row) per
    // warp at a time, the finisher's first.
    auto help_merge = [&]() {
        if (!__all_sync(0xffffffffu, mbar_wait(&settle_bar, 0, abort_flag))) return;
        const uint32_t nl = s_nlast;
        for (uint32_t pr = warp == FINISH ? 0u : (uint32_t)warp + 1u; pr < nl * rep; pr += FINISH + 1) {
            const uint32_t k = pr / rep;
            lean_merge_row<HD, NQ>(P, U, pend[k][0], pend[k][1], pend[k][2], pend[k][3], (int)(pr % rep), lane);
        }
    };

    if (warp == PRODUCER) {
        // ---------------- units -> segment descriptors + TMA boxes (one lane)
        if (lane == 0) {
            if (!P.early_kv) grid_dep_wait();
            uint32_t u = blockIdx.x, seg = 0, tc = 0;
            const int na = (int)P.lean_ahead;
            // The first dynamic units are taken once the first wave of boxes
            // is in flight: at launch every CTA's grab hits one counter, and
            // the first boxes need not wait for that.
            uint32_t ahead[kLeanAheadMax];
            bool grabbed = false;
#define ND_LEAN_GRAB_AHEAD()                                                                        \
    do {                                                                                            \
        _Pragma("unroll") for (int a = 0; a < kLeanAheadMax; a++)                                  \
            ahead[a] = a < na && U.NU > U.G ? (uint32_t)atomicAdd(work_ctr, 1) + U.G : U.NU;       \
        grabbed = true;                                                                             \
    } while (0)
#pragma unroll
            for (int a = 0; a < kLeanAheadMax; a++) ahead[a] = U.NU;
            while (u < U.NU && !*abort_flag) {
                uint32_t x = U.start(u);
                const uint32_t xe = U.start(u + 1);
                LeanWalk w;
                if (tk.n) w.init_at(tk.tok, tk.n, x);
                else w.init(P, u);
                while (x < xe && !*abort_flag) {
                    const uint32_t nt = min(xe - x, w.T - w.kt), i = seg % SQ;
                    if (seg >= SQ && !mbar_wait(&slot_free[i], ((seg / SQ) - 1) & 1, abort_flag)) break;
                    desc[i] = LeanDesc{w.t, w.g, w.kt, nt, w.T, w.item_start(), u, 0u, w.seq, w.pos};
                    mbar_arrive(&desc_full[i]);
                    // The first query rows load while the memory system is idle:
                    // behind the first wave of boxes they would take the loaded
                    // latency (several us) and hold every consumer back.
                    if (seg == 0 && !P.early_kv && !mbar_wait(&q_full[0], 0, abort_flag)) break;
                    for (uint32_t k2 = 0; k2 < nt; k2++, tc++) {
                        const int y = (int)phys_row(P.c, w.seq, (w.kt + k2) * TR);
                        const uint32_t s2 = tc % STAGES;
                        if (tc == STAGES && !grabbed) ND_LEAN_GRAB_AHEAD();
                        if (tc >= STAGES && !mbar_wait(&empty[s2], ((tc / STAGES) - 1) & 1, abort_flag)) break;
                        // Rows of this tile the item reads: [row0, jw). A tile that
                        // ends 16 or more rows past them takes 16-row sub-boxes (the
                        // rest of the stage keeps stale rows, which the consumers mask).
                        const uint32_t row0 = (w.kt + k2) * TR, jw = w.pos + 1u - (P.fuse_append ? 1u : 0u);
                        const uint32_t nsub = jw >= row0 + (uint32_t)(TR - C::SUBR) + 1u
                                                  ? 0u
                                                  : jw > row0 ? (jw - row0 + C::SUBR - 1) / C::SUBR : 1u;
                        mbar_expect_tx(&full[s2], (nsub ? 2 * nsub * C::SUB : 2 * TILE_BYTES) + 2 * C::SC);
                        if (nsub == 0) {
                            tma_load_2d(smem + s2 * TILE_BYTES, &kmap, (int)(w.g * HD), y, &full[s2]);
                            tma_load_2d(smem + C::OFF_V + s2 * TILE_BYTES, &vmap, (int)(w.g * HD), y, &full[s2]);
                        } else {
                            for (uint32_t j = 0; j < nsub; j++) {
                                const int yj = y + (int)j * C::SUBR;
                                tma_load_2d(smem + s2 * TILE_BYTES + j * C::SUB, &ktmap, (int)(w.g * HD), yj,
                                            &full[s2]);
                                tma_load_2d(smem + C::OFF_V + s2 * TILE_BYTES + j * C::SUB, &vtmap,
                                            (int)(w.g * HD), yj, &full[s2]);
                            }
                        }
                        if constexpr (C::I8) {   // x = the KV head rounded down to a multiple of 4 (16 bytes)
                            tma_load_2d(smem + C::OFF_KS + s2 * C::SC, &ksmap, (int)(w.g & ~3u), y, &full[s2]);
                            tma_load_2d(smem + C::OFF_VS + s2 * C::SC, &vsmap, (int)(w.g & ~3u), y, &full[s2]);
                        }
                    }
                    x += nt;
                    w.advance(P, nt);
                    seg++;
                }
                if (!grabbed) ND_LEAN_GRAB_AHEAD();
                u = ahead[0];
#pragma unroll
                for (int a = 0; a + 1 < kLeanAheadMax; a++) ahead[a] = ahead[a + 1];
                const uint32_t grab = u < U.NU ? (uint32_t)atomicAdd(work_ctr, 1) + U.G : U.NU;
#pragma unroll
                for (int a = 0; a < kLeanAheadMax; a++)
                    if (a == na - 1) ahead[a] = grab;
            }
#undef ND_LEAN_GRAB_AHEAD
            // Every unit taken must be counted before the stop lets the finisher
            // report this CTA done (the last CTA out rewinds the counter): wait
            // for the values of the grabs still in flight.
            uint32_t pending = 0;
#pragma unroll
            for (int a = 0; a < kLeanAheadMax; a++) pending |= ahead[a];
            if (!*abort_flag) {
                const uint32_t i = seg % SQ;
                if (seg < SQ || mbar_wait(&slot_free[i], ((seg / SQ) - 1) & 1, abort_flag)) {
                    desc[i] = LeanDesc{0u, 0u, 0u, 0u, 1u, 0u, pending, 1u, 0u, 0u};   // storing pending waits for the grabs
                    mbar_arrive(&desc_full[i]);
                }
            }
            if (*abort_flag && tc) mbar_drain(&full[(tc - 1) % STAGES], ((tc - 1) / STAGES) & 1);
        }
        __syncwarp();
        help_merge();
        return;
    }

    if (warp == PREP) {
        // ---------------- query rows and the fused append of each segment
        grid_dep_wait();
        if (lane == 0) grid_dep_launch();
        for (uint32_t seg = 0;; seg++) {
            const uint32_t i = seg % SQ;
            if (!__all_sync(0xffffffffu, mbar_wait(&desc_full[i], (seg / SQ) & 1, abort_flag))) return;
            const LeanDesc d = desc[i];
            if (d.stop) {
                help_merge();
                return;
            }
            const TokMeta tm{d.seq, 0u, d.t};
            const uint32_t pos = d.pos;
            const bool bad = pos >= P.max_pos || pos >= W;   // the host routes only non-wrapping calls here
            const uint32_t pr = bad ? 0u : pos;
            const float2 *cs = P.rope + (size_t)pr * (HD / 2);
            const bool appender = !bad && P.fuse_append && d.kt + d.nt == d.T;
            // All query rows and this lane's (cos, sin) pairs in one load round.
            constexpr int PPL = RopePairs<HD>::PPL;
            RopePairs<HD> xs[NQ];
            float2 csv[PPL];
#pragma unroll
            for (int cc = 0; cc < PPL; cc++) {
                const int k2 = lane + 32 * cc;
                csv[cc] = k2 < HD / 2 ? cs[k2] : make_float2(0.0f, 0.0f);
            }
#pragma unroll
            for (int qi = 0; qi < NQ; qi++) {
                if (qi < (int)rep && !bad)
                    warp_load_pairs<HD>(xs[qi], P.q, P.act_dt, ((size_t)tm.row * P.n_heads + d.g * rep + qi) * HD,
                                        lane);
            }
#pragma unroll
            for (int qi = 0; qi < NQ; qi++) {
                if (qi < (int)rep && !bad) {
                    warp_norm_rope_v<HD>(xs[qi], csv, P.qnorm, lane);
#pragma unroll
                    for (int cc = 0; cc < PPL; cc++) {
                        const int k2 = lane + 32 * cc;
                        if (k2 < HD / 2) {
                            sq[i][qi][k2] = xs[qi].a[cc] * P.scale_log2;
                            sq[i][qi][k2 + HD / 2] = xs[qi].b[cc] * P.scale_log2;
                        }
                    }
                } else {
                    for (int k2 = lane; k2 < HD; k2 += 32) sq[i][qi][k2] = 0.0f;
                }
            }
            if (lane == 0) {
                if (bad) set_err(P.err, 2);
                info[i] = LeanInfo{tm.row, pr, bad ? 0u : pos + 1 - (P.fuse_append ? 1u : 0u), tm.seq,
                                   appender ? 1 : 0};
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&q_full[i]);
            // The newest row is read only at the end of the segment: append it
            // after releasing the queries, and signal it on its own barrier.
            if (appender)
                warp_append<HD, HD, KVT>(P.c, phys_row(P.c, tm.seq, pos), d.g, P.k, P.v, P.act_dt,
                                         ((size_t)tm.row * n_kv + d.g) * HD, ((size_t)tm.row * n_kv + d.g) * HD, cs,
                                         P.knorm, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&app_full[i]);
        }
    }

    if (warp == FINISH) {
        // ---------------- merge of the four consumer warps: output or partial
        grid_dep_wait();
        uint32_t npend = 0;
        // Tickets of the pieces noted so far (one fence, one atomic per lane);
        // the items whose last piece this was move to the front of pend.
        auto settle = [&]() -> uint32_t {
            __threadfence();
            __syncwarp();
            bool last = false;
            uint32_t key = 0, e0 = 0, e1 = 0, e2 = 0, e3 = 0;
            if (lane < (int)npend) {
                e0 = pend[lane][0], e1 = pend[lane][1], e2 = pend[lane][2], e3 = pend[lane][3];
                key = U.unit_of(e0);
                last = atomicAdd(&P.counters[key], 1) == (int)(U.unit_of(e0 + e1 - 1) - key);
            }
            const uint32_t msk = __ballot_sync(0xffffffffu, last);
            __syncwarp();
            if (last) {
                const uint32_t k = __popc(msk & ((1u << lane) - 1u));
                pend[k][0] = e0, pend[k][1] = e1, pend[k][2] = e2, pend[k][3] = e3;
                P.counters[key] = 0;
            }
            if (msk) __threadfence();
            __syncwarp();
            npend = 0;
            return (uint32_t)__popc(msk);
        };
        for (uint32_t seg = 0;; seg++) {
            const uint32_t i = seg % SQ, par = (seg / SQ) & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&desc_full[i], par, abort_flag))) break;
            const LeanDesc d = desc[i];
            if (d.stop) {
                const uint32_t nl = npend ? settle() : 0u;
                // Last CTA out rewinds the unit counter for the next launch
                // (every CTA has taken its final unit before its stop).
                if (lane == 0 && U.NU > U.G && atomicAdd(done_ctr, 1) == (int)U.G - 1) {
                    *work_ctr = 0;
                    *done_ctr = 0;
                }
                if (lane == 0) {
                    s_nlast = nl;
                    mbar_arrive(&settle_bar);   // the other warps merge with this one
                }
                help_merge();
                break;
            }
            if (!__all_sync(0xffffffffu, mbar_wait(&q_full[i], par, abort_flag))) break;
            if (!__all_sync(0xffffffffu, mbar_wait(&mb_full[i], par, abort_flag))) break;
            const uint32_t row = info[i].row;
            const uint32_t uf = U.unit_of(d.istart), ul = U.unit_of(d.istart + d.T - 1);
            const uint32_t nsplit = ul - uf + 1;
            const size_t out_base = (size_t)row * P.n_heads;
            const uint32_t slot = 2 * d.unit + (d.istart > U.start(d.unit) ? 1u : 0u);
            for (int idx = lane; idx < (int)rep * HD; idx += 32) {
                const int qi = idx / HD, e = idx % HD;
                float M = mml[i][0][qi][0];
#pragma unroll
                for (int w2 = 1; w2 < NW; w2++) M = fmaxf(M, mml[i][w2][qi][0]);
                float o = 0.0f, L = 0.0f;
#pragma unroll
                for (int w2 = 0; w2 < NW; w2++) {
                    const float f = ex2(mml[i][w2][qi][0] - M);
                    o += mo[i][w2][qi][e] * f;
                    L += mml[i][w2][qi][1] * f;
                }
                if (nsplit == 1) {
                    const uint32_t h = d.g * rep + qi;
                    float val = o / L;
                    if (P.gate)
                        val *= 1.0f / (1.0f + ex2(-act_load(P.gate, P.act_dt, (out_base + h) * HD + e) *
                                                  1.4426950408889634f));
                    out_store<HD>(P, row, h * HD + e, val);
                } else {
                    P.part_o[((size_t)slot * NQ + qi) * HD + e] = o;
                    if (e == 0) {
                        P.part_ml[((size_t)slot * NQ + qi) * 2 + 0] = M;
                        P.part_ml[((size_t)slot * NQ + qi) * 2 + 1] = L;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&slot_free[i]);
            if (nsplit > 1) {
                if (lane == 0) {
                    pend[npend][0] = d.istart;
                    pend[npend][1] = d.T;
                    pend[npend][2] = d.g;
                    pend[npend][3] = row;
                }
                __syncwarp();
                if (++npend == 32) {   // rare: the finisher alone merges what completed
                    const uint32_t nl = settle();
                    for (uint32_t pr = 0; pr < nl * rep; pr++)
                        lean_merge_row<HD, NQ>(P, U, pend[pr / rep][0], pend[pr / rep][1], pend[pr / rep][2],
                                               pend[pr / rep][3], (int)(pr % rep), lane);
                    __syncwarp();
                }
            }
        }
        if (lane == 0 && abort_flag_s) set_err(P.err, 3);
        return;
    }

    // ---------------- consumers (warps 0..NW-1)
    const int sub = lane % LPR, rl = lane / LPR;
    float zero_sc[UB];
#pragma unroll
    for (int u = 0; u < UB; u++) zero_sc[u] = 0.0f;
    uint32_t tc = 0;
    for (uint32_t seg = 0;; seg++) {
        const uint32_t i = seg % SQ, par = (seg / SQ) & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&desc_full[i], par, abort_flag))) return;
        const LeanDesc d = desc[i];
        if (d.stop) {
            help_merge();
            return;
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&q_full[i], par, abort_flag))) return;
        float qr[NQ][EK];
#pragma unroll
        for (int qi = 0; qi < NQ; qi++)
#pragma unroll
            for (int e = 0; e < EK; e++) qr[qi][e] = sq[i][qi][sub * EK + e];
        const LeanInfo si = info[i];
        uint32_t ql[NQ][3][C::I8 ? EK / 4 : 1];
        float cq[NQ][3];
        if constexpr (C::I8) q_limbs<NQ, EK, LPR>(qr, ql, cq);

        float m[NQ], l[NQ], acc[NQ][EV];
#pragma unroll
        for (int qi = 0; qi < NQ; qi++) {
            m[qi] = -INFINITY;
            l[qi] = 0.0f;
#pragma unroll
            for (int e = 0; e < EV; e++) acc[qi][e] = 0.0f;
        }
        const uint32_t jb = d.kt * TR;
        for (uint32_t k2 = 0; k2 < d.nt; k2++, tc++) {
            const uint32_t s2 = tc % STAGES;
            if (!__all_sync(0xffffffffu, mbar_wait(&full[s2], (tc / STAGES) & 1, abort_flag))) return;
            const uint8_t *kt = smem + s2 * TILE_BYTES, *vt = smem + C::OFF_V + s2 * TILE_BYTES;
#pragma unroll
            for (int cI = 0; cI < NCALL; cI++) {
                uint32_t kw[UB][WK], vw[UB][WV];
                bool valid[UB];
#pragma unroll
                for (int u = 0; u < UB; u++) {
                    const int r = warp * RW + (cI * UB + u) * RPW + rl;   // row within the tile
                    valid[u] = jb + k2 * TR + r < si.jend;
                    const uint32_t *kp = reinterpret_cast<const uint32_t *>(kt + r * HD * ES + sub * EK * ES);
                    const uint32_t *vp = reinterpret_cast<const uint32_t *>(vt + r * HD * ES + sub * EV * ES);
#pragma unroll
                    for (int k3 = 0; k3 < WK; k3++) kw[u][k3] = kp[k3];
#pragma unroll
                    for (int k3 = 0; k3 < WV; k3++) vw[u][k3] = valid[u] ? vp[k3] : 0u;   // 0 * (Inf|NaN) guard
                }
                if constexpr (C::I8) {
                    // The rows' scales (column g & 3 of the stage's {4, 64} box);
                    // a row past the item's end gets scale 0, so stale or NaN
                    // scale bits contribute nothing.
                    const float *ks = reinterpret_cast<const float *>(smem + C::OFF_KS + s2 * C::SC);
                    const float *vs = reinterpret_cast<const float *>(smem + C::OFF_VS + s2 * C::SC);
                    float ksc[UB], vsc[UB];
#pragma unroll
                    for (int u = 0; u < UB; u++) {
                        const int r = warp * RW + (cI * UB + u) * RPW + rl;
                        ksc[u] = valid[u] ? ks[r * 4 + (d.g & 3u)] : 0.0f;
                        vsc[u] = valid[u] ? vs[r * 4 + (d.g & 3u)] : 0.0f;
                    }
                    float sc[UB][NQ];
                    qk_i8dp<NQ, EK, UB>(ql, cq, kw, sc);
                    consume_scores<HD, HD, KVT, NQ, UB, true>(sc, vw, ksc, vsc, valid, m, l, acc);
                } else {
                    consume<HD, HD, KVT, NQ, UB>(qr, kw, vw, zero_sc, zero_sc, valid, m, l, acc);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s2]);
        }
        if (si.appender && warp == NW - 1) {
            // The newest row, written by the prep warp (app_full): plain
            // coherent loads, not TMA.
            if (!__all_sync(0xffffffffu, mbar_wait(&app_full[i], par, abort_flag))) return;
            const char *kb = static_cast<const char *>(P.c.k) + ((size_t)d.g * HD + (size_t)sub * EK) * ES;
            const char *vb = static_cast<const char *>(P.c.v) + ((size_t)d.g * HD + (size_t)sub * EV) * ES;
            const size_t row = phys_row(P.c, si.seq, si.pos);
            uint32_t kw[1][WK], vw[1][WV];
            float ksc1[1] = {0.0f}, vsc1[1] = {0.0f};
            if constexpr (C::I8) {   // its scales, written by the same launch: coherent loads too
                ksc1[0] = *reinterpret_cast<const volatile float *>(P.c.ks + row * P.c.n_kv + d.g);
                vsc1[0] = *reinterpret_cast<const volatile float *>(P.c.vs + row * P.c.n_kv + d.g);
            }
            const bool valid[1] = {rl == 0};
            load_words<WK, false>(kb + row * (size_t)P.c.k_dim * ES, kw[0]);
            load_words<WV, false>(vb + row * (size_t)P.c.v_dim * ES, vw[0]);
            if constexpr (C::I8) {
                float sc1[1][NQ];
                qk_i8dp<NQ, EK, 1>(ql, cq, kw, sc1);
                consume_scores<HD, HD, KVT, NQ, 1, true>(sc1, vw, ksc1, vsc1, valid, m, l, acc);
            } else {
                consume<HD, HD, KVT, NQ, 1, true>(qr, kw, vw, ksc1, vsc1, valid, m, l, acc);
            }
        }
        // Reduce across the row lanes; hand (m, l, acc) of this warp over.
#pragma unroll
        for (int qi = 0; qi < NQ; qi++) {
#pragma unroll
            for (int o = LPR; o < 32; o <<= 1) {
                l[qi] += __shfl_xor_sync(0xffffffffu, l[qi], o);
#pragma unroll
                for (int e = 0; e < EV; e++) acc[qi][e] += __shfl_xor_sync(0xffffffffu, acc[qi][e], o);
            }
        }
        if (rl == 0) {
#pragma unroll
            for (int qi = 0; qi < NQ; qi++)
#pragma unroll
                for (int e = 0; e < EV; e++) mo[i][warp][qi][sub * EV + e] = acc[qi][e];
        }
        if (lane == 0) {
#pragma unroll
            for (int qi = 0; qi < NQ; qi++) {
                mml[i][warp][qi][0] = m[qi];
                mml[i][warp][qi][1] = l[qi];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&mb_full[i]);
    }
}

}  // namespace nda
