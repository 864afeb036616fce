// nd_device.cuh - device side of the Needle attention hot path for sm_100a.
//
// Kernels (one template family each):
//   append_kernel   K1: per (token, KV head) warp: optional ZC-RMSNorm + NeoX
//                   RoPE of k, then the KV store at kv_slot(pos) (int8+scale,
//                   f32, f16 or bf16). Reference: zcrms_head_rows
//                   (engine/src/nd_model.c:326-365), the store loop of
//                   attention() (nd_model.c:2426-2449), kv_store_int8
//                   (nd_model.c:1822-1866), kv_slot (nd_model.c:1304-1309).
//   attend_kernel   K3+K4: split-KV ("flash-decoding") attention of one query
//                   token's GQA group over the sink run and the recent run
//                   (nd_model.c:2451-2481, attn_heads 2105-2359), 128-bit
//                   coalesced KV loads, warp-shuffle reductions, online softmax
//                   in the log2 domain; splits merged by the last CTA to finish
//                   (atomic ticket, no spin), sigmoid gate fused on the emit
//                   (attn_gate_emit, nd_model.c:2091-2103). With fuse_append the
//                   CTA that owns the newest position also runs K1 for it.
//
// Bit-exactness contract: the rotated K and every int8 byte/scale equal the
// reference's, so the fp32 RoPE arithmetic below uses explicitly rounded
// intrinsics (no FMA contraction) in the reference's statement order, the
// cos/sin come from a table the host builds with the reference's own
// expressions, and the int8 quotient is formed the way kv_store_int8 forms it.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <type_traits>

namespace nda {

enum : int { DT_I8 = 0, DT_F32 = 1, DT_F16 = 2, DT_BF16 = 3 };

// Rows per TMA box of the TMA-staged decode kernels (16-bit caches); a tile of
// the balanced kernel is one box, its splits are multiples.
constexpr int kTmaRows = 64;
// int8 tiles of the balanced kernel take 128 rows. One lane issues every TMA
// box, and a box costs its issue about the same whatever its bytes, so int8's
// half-size rows (and its two scale boxes per tile) would leave that lane the
// limit at 64 rows.
constexpr int kLeanRowsI8 = 128;
constexpr int lean_rows(bool i8) { return i8 ? kLeanRowsI8 : kTmaRows; }

// Per-sequence session state (nd_model.h:130-131: pos, n_sink).
struct SeqState {
    uint32_t pos, n_sink;
};

// One query token of a call: its sequence, its offset from the sequence's
// current position, and its row in the packed q/k/v/gate/out tensors.
struct TokMeta {
    uint32_t seq, off, row;
};

// One sequence of a batched prefill call: its tokens are rows
// [tok_base, tok_base + len) of the packed tensors, in position order.
struct SeqSpan {
    uint32_t seq, tok_base, len;
};

// One layer of the cache. Rows are [n_kv][head_dim] elements; a sequence's
// logical slot s lives in row seq*window + s (contiguous) or in page
// btab[seq][s >> block_shift] at offset s & mask (paged).
struct CacheView {
    void *k, *v;
    float *ks, *vs;              // int8 scales [row][n_kv]
    uint32_t k_dim, v_dim, n_kv, window;
    const int32_t *btab;         // nullptr = contiguous
    uint32_t blocks_per_seq, block_shift;
    int *vbig;                   // bf16 caches: the layer's flag "K or V holds a value f16 cannot represent"
};

// A bf16 pair word holding a value with |x| >= 2^16, Inf or NaN (exponent
// field >= 143): values f16 cannot represent. Writers of a bf16 cache set the
// layer's flag when they store one in K or V (the tensor-core prefill converts
// K and V tiles to f16 only while the flag is clear).
__device__ __forceinline__ bool bf16x2_big(uint32_t w) {
    return (w & 0x7f80u) >= 0x4780u || (w & 0x7f800000u) >= 0x47800000u;
}

// Head-sharded decode (G ranks, one GPU each, every rank holding the same
// sequences for its own KV heads): the attend kernels store each output row
// straight into this call's gather slot on every rank (peer memory over
// NVLink, the own rank included), rows of row_elems elements with this rank's
// heads at column col0. The slot holds 8-byte words {4 bytes of output (one
// f32 or two 16-bit elements), the call's epoch}, each written by one 64-bit
// store, so a reader knows a word has arrived when it carries the epoch: no
// fence and no flag are needed. G = 0: plain output to out.
constexpr int kMaxGather = 8;
struct GatherView {
    unsigned long long *slot[kMaxGather];    // this call's slot in rank p's gather buffer
    uint32_t G, col0, row_elems, epoch;
};

struct AttnParams {
    const void *q, *k, *v, *gate;
    void *out;
    GatherView gth;
    int act_dt, out_dt;
    CacheView c;
    const float2 *rope;          // [max_pos][qk_hd/2] (cos, sin)
    uint32_t max_pos;
    const float *qnorm, *knorm;  // [qk_hd] or nullptr
    const SeqState *state;
    const TokMeta *tok;          // per-token map, or
    const SeqSpan *spans;        // per-sequence spans (binary search), or neither:
    uint32_t n_spans;            //   token i = sequence i, offset 0, row i
    uint32_t n_tok, n_heads, rep;
    float scale_log2;            // log2(e) / sqrtf(qk_hd)
    uint32_t chunk;              // visit rows per split (implicit grid)
    uint32_t max_splits;         // split stride of the scratch
    const uint32_t *split_cu;    // exact grid: prefix sum of splits per token (n_tok+1), or nullptr;
                                 //   balanced grid: n_kv x prefix sum of 64-row tiles per token
    const uint32_t *cta_tok;     // balanced grid: token holding each unit's first tile
    uint32_t n_cta, n_tiles;     // balanced grid: CTAs, tiles of the call
    uint32_t lean_s, lean_ch;    // balanced grid: tiles per static unit, per dynamic unit
    uint32_t n_units, work_slot; // balanced grid: units; counters[work_slot..+1] = unit / done counters
    uint32_t lean_ahead;         // balanced grid: dynamic units a producer holds ahead (1..4)
    int early_kv;                // balanced grid: K/V may be streamed before the previous kernel ends
    int fuse_append;
    float *part_o, *part_ml;
    int *counters;
    int *err;                    // status word in mapped pinned host memory (0 = ok)
};

// Balanced decode of a call of at most kLeanParamTok tokens: the plan's token
// table travels as a kernel parameter, so no host-to-device copy sits between
// consecutive launches.
constexpr int kLeanParamTok = 128;
struct LeanTok {
    uint32_t n;                       // tokens in tok; 0: the plan is in global memory
    uint32_t pad[3];
    uint4 tok[kLeanParamTok + 1];     // per token {first tile, tiles per item, sequence, position};
                                      //   entry n: {tiles of the call, 0, 0, 0}
};

// ---------------------------------------------------------------- helpers
// The status word is host memory mapped into the device's address space, so
// the host reads it after a stream sync with no copy. A plain store: any
// nonzero code fails the call, and racing writers need no atomicity.
__device__ __forceinline__ void set_err(int *err, int code) { *reinterpret_cast<volatile int *>(err) = code; }

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float act_load(const void *p, int dt, size_t i) {
    if (dt == DT_F32) return static_cast<const float *>(p)[i];
    if (dt == DT_F16) return __half2float(static_cast<const __half *>(p)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
}

__device__ __forceinline__ void act_store(void *p, int dt, size_t i, float x) {
    if (dt == DT_F32) static_cast<float *>(p)[i] = x;
    else if (dt == DT_F16) static_cast<__half *>(p)[i] = __float2half_rn(x);
    else static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(x);
}

// Output element (row, col) of a call, col = head * VD + d over this
// launch's heads: into out, or (head-sharded) into every rank's gather slot
// at the rank's column offset. Head-sharded with 16-bit outputs, the whole
// warp calls this together with consecutive cols in consecutive lanes (col
// parity = lane parity): the even lane stores the pair. Static indices over
// the rank list keep the parameter array out of local memory.
template <int VD>
__device__ __forceinline__ void out_store(const AttnParams &P, size_t row, uint32_t col, float x) {
    if (P.gth.G == 0) {
        act_store(P.out, P.out_dt, row * P.n_heads * VD + col, x);
        return;
    }
    const size_t e = row * P.gth.row_elems + P.gth.col0 + col;   // element of the gathered rows
    uint32_t data;
    size_t wi;
    if (P.out_dt == DT_F32) {
        data = __float_as_uint(x);
        wi = e;
    } else {
        const float y = __shfl_xor_sync(0xffffffffu, x, 1);
        if (col & 1u) return;
        if (P.out_dt == DT_F16) {
            const __half2 t = __floats2half2_rn(x, y);
            data = *reinterpret_cast<const uint32_t *>(&t);
        } else {
            const __nv_bfloat162 t = __floats2bfloat162_rn(x, y);
            data = *reinterpret_cast<const uint32_t *>(&t);
        }
        wi = e >> 1;
    }
    const unsigned long long w = ((unsigned long long)P.gth.epoch << 32) | data;
#pragma unroll
    for (int p = 0; p < kMaxGather; p++)
        if ((uint32_t)p < P.gth.G)
            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(P.gth.slot[p] + wi), "l"(w) : "memory");
}

__device__ __forceinline__ TokMeta token_meta(const AttnParams &P, uint32_t tok) {
    if (P.tok) return P.tok[tok];
    if (P.spans) {
        uint32_t lo = 0, hi = P.n_spans;   // last span with tok_base <= tok
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) >> 1;
            if (P.spans[mid].tok_base <= tok) lo = mid;
            else hi = mid;
        }
        return TokMeta{P.spans[lo].seq, tok - P.spans[lo].tok_base, tok};
    }
    return TokMeta{tok, 0u, tok};
}

__device__ __forceinline__ uint32_t kv_slot(uint32_t window, uint32_t n_sink, uint32_t p) {
    return p < n_sink ? p : n_sink + (p - n_sink) % (window - n_sink);
}

__device__ __forceinline__ size_t phys_row(const CacheView &c, uint32_t seq, uint32_t slot) {
    if (c.btab) {
        const uint32_t mask = (1u << c.block_shift) - 1u;
        const size_t page = (size_t)c.btab[(size_t)seq * c.blocks_per_seq + (slot >> c.block_shift)];
        return (page << c.block_shift) | (slot & mask);
    }
    return (size_t)seq * c.window + slot;
}

// The visited positions of a token at `pos`: sinks [0, sinks), then the recent
// run [rfirst, rfirst + rcount) (nd_model.c:2456-2477). Visit index j maps to
// a slot without a modulo per row: recent slots are consecutive in the ring.
struct Runs {
    uint32_t sinks, rfirst, rcount, r0slot;
};

__device__ __forceinline__ Runs make_runs(uint32_t pos, uint32_t n_sink, uint32_t window) {
    Runs r;
    r.sinks = n_sink < pos + 1 ? n_sink : pos + 1;
    if (pos + 1 <= n_sink) {
        r.rfirst = pos + 1;
        r.rcount = 0;
    } else {
        r.rcount = pos + 1 - n_sink;
        if (r.rcount > window - n_sink) r.rcount = window - n_sink;
        r.rfirst = pos + 1 - r.rcount;
    }
    r.r0slot = r.rcount ? kv_slot(window, n_sink, r.rfirst) : 0;
    return r;
}

__device__ __forceinline__ uint32_t visit_slot(const Runs &r, uint32_t j, uint32_t n_sink,
                                               uint32_t window) {
    if (j < r.sinks) return j;
    const uint32_t s = r.r0slot + (j - r.sinks);
    return s >= window ? s - (window - n_sink) : s;
}

// Symmetric int8 code of x for a row scale: the quotient is formed as
// kv_store_int8 forms it (nd_model.c:1856-1865: r = RN(1/scale), q = RN(x*r),
// residual e = fma(-scale, q, x), q = fma(e, r, q) - the correctly rounded
// quotient for finite rows; a plain divide outside +-1e30), clamped to +-127
// and rounded half to even like lrintf.
__device__ __forceinline__ int8_t q8(float x, float scale, float r) {
    float q;
    if (x > -1e30f && x < 1e30f) {
        q = __fmul_rn(x, r);
        const float e = __fmaf_rn(-scale, q, x);
        q = __fmaf_rn(e, r, q);
    } else {
        q = __fdiv_rn(x, scale);
    }
    if (q > 127.0f) q = 127.0f;
    if (q < -127.0f) q = -127.0f;
    return (int8_t)__float2int_rn(q);
}

template <typename KVT> struct KvT;
template <> struct KvT<int8_t> { static constexpr int dt = DT_I8; };
template <> struct KvT<float> { static constexpr int dt = DT_F32; };
template <> struct KvT<__half> { static constexpr int dt = DT_F16; };
template <> struct KvT<__nv_bfloat16> { static constexpr int dt = DT_BF16; };

template <typename KVT> __device__ __forceinline__ KVT kv_from_float(float x);
template <> __device__ __forceinline__ float kv_from_float<float>(float x) { return x; }
template <> __device__ __forceinline__ __half kv_from_float<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 kv_from_float<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

// ------------------------------------------------- warp-level norm + RoPE
// One head row of QK values held as rotation pairs: lane handles pair index
// i = lane + 32*c (c < PPL), with a = x[i], b = x[i + QK/2]. The squared sum
// of the norm is accumulated in index order 0..QK-1 by every lane (values are
// broadcast by shuffles), matching zcrms_head_rows' sequential loop.
template <int QK>
struct RopePairs {
    static constexpr int HALF = QK / 2;
    static constexpr int PPL = (HALF + 31) / 32;
    float a[PPL], b[PPL];
};

template <int QK>
__device__ __forceinline__ void warp_norm_rope(RopePairs<QK> &x, const float2 *cs,
                                               const float *norm, int lane) {
    constexpr int HALF = QK / 2;
    constexpr int PPL = RopePairs<QK>::PPL;
    static_assert(QK % 2 == 0, "even head dim");
    if (norm) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < QK; i++) {
            const int ii = i < HALF ? i : i - HALF;
            const float xi = i < HALF ? __shfl_sync(0xffffffffu, x.a[ii / 32], ii % 32)
                                      : __shfl_sync(0xffffffffu, x.b[ii / 32], ii % 32);
            ss = __fadd_rn(ss, __fmul_rn(xi, xi));
        }
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)QK), 1e-6f)));
#pragma unroll
        for (int c = 0; c < PPL; c++) {
            const int i = lane + 32 * c;
            if (i < HALF) {
                x.a[c] = __fmul_rn(__fmul_rn(__fadd_rn(1.0f, norm[i]), x.a[c]), inv);
                x.b[c] = __fmul_rn(__fmul_rn(__fadd_rn(1.0f, norm[i + HALF]), x.b[c]), inv);
            }
        }
    }
#pragma unroll
    for (int c = 0; c < PPL; c++) {
        const int i = lane + 32 * c;
        if (i < HALF) {
            const float2 t = cs[i];
            const float a = x.a[c], b = x.b[c];
            x.a[c] = __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(b, t.y));
            x.b[c] = __fadd_rn(__fmul_rn(b, t.x), __fmul_rn(a, t.y));
        }
    }
}

// Same, with this lane's (cos, sin) pairs already loaded: csv[c] belongs to
// pair lane + 32 c.
template <int QK>
__device__ __forceinline__ void warp_norm_rope_v(RopePairs<QK> &x, const float2 (&csv)[RopePairs<QK>::PPL],
                                                 const float *norm, int lane) {
    constexpr int HALF = QK / 2;
    constexpr int PPL = RopePairs<QK>::PPL;
    static_assert(QK % 2 == 0, "even head dim");
    if (norm) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < QK; i++) {
            const int ii = i < HALF ? i : i - HALF;
            const float xi = i < HALF ? __shfl_sync(0xffffffffu, x.a[ii / 32], ii % 32)
                                      : __shfl_sync(0xffffffffu, x.b[ii / 32], ii % 32);
            ss = __fadd_rn(ss, __fmul_rn(xi, xi));
        }
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)QK), 1e-6f)));
#pragma unroll
        for (int c = 0; c < PPL; c++) {
            const int i = lane + 32 * c;
            if (i < HALF) {
                x.a[c] = __fmul_rn(__fmul_rn(__fadd_rn(1.0f, norm[i]), x.a[c]), inv);
                x.b[c] = __fmul_rn(__fmul_rn(__fadd_rn(1.0f, norm[i + HALF]), x.b[c]), inv);
            }
        }
    }
#pragma unroll
    for (int c = 0; c < PPL; c++) {
        const int i = lane + 32 * c;
        if (i < HALF) {
            const float2 t = csv[c];
            const float a = x.a[c], b = x.b[c];
            x.a[c] = __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(b, t.y));
            x.b[c] = __fadd_rn(__fmul_rn(b, t.x), __fmul_rn(a, t.y));
        }
    }
}

template <int QK>
__device__ __forceinline__ void warp_load_pairs(RopePairs<QK> &x, const void *src, int dt,
                                                size_t base, int lane) {
    constexpr int HALF = QK / 2;
#pragma unroll
    for (int c = 0; c < RopePairs<QK>::PPL; c++) {
        const int i = lane + 32 * c;
        x.a[c] = i < HALF ? act_load(src, dt, base + i) : 0.0f;
        x.b[c] = i < HALF ? act_load(src, dt, base + i + HALF) : 0.0f;
    }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// K1 for one (token, KV head g): rotate k, store k and v at physical row `row`.
template <int QK, int VD, typename KVT>
__device__ __forceinline__ void warp_append(const CacheView &c, size_t row, uint32_t g,
                                            const void *k, const void *v, int act_dt,
                                            size_t krow_base, size_t vrow_base,
                                            const float2 *cs, const float *knorm, int lane) {
    constexpr int HALF = QK / 2;
    constexpr int VPL = (VD + 31) / 32;
    RopePairs<QK> kx;
    warp_load_pairs<QK>(kx, k, act_dt, krow_base, lane);
    float vx[VPL];
#pragma unroll
    for (int cI = 0; cI < VPL; cI++) {
        const int i = lane + 32 * cI;
        vx[cI] = i < VD ? act_load(v, act_dt, vrow_base + i) : 0.0f;
    }
    warp_norm_rope<QK>(kx, cs, knorm, lane);
    const size_t kbase = row * c.k_dim + (size_t)g * QK;
    const size_t vbase = row * c.v_dim + (size_t)g * VD;
    if constexpr (KvT<KVT>::dt == DT_I8) {
        float mk = 0.0f, mv = 0.0f;
#pragma unroll
        for (int cI = 0; cI < RopePairs<QK>::PPL; cI++)
            mk = fmaxf(mk, fmaxf(fabsf(kx.a[cI]), fabsf(kx.b[cI])));
#pragma unroll
        for (int cI = 0; cI < VPL; cI++) mv = fmaxf(mv, fabsf(vx[cI]));
        mk = warp_max(mk);
        mv = warp_max(mv);
        const float ksc = mk > 0.0f ? __fdiv_rn(mk, 127.0f) : 1.0f;
        const float vsc = mv > 0.0f ? __fdiv_rn(mv, 127.0f) : 1.0f;
        const float kr = __fdiv_rn(1.0f, ksc), vr = __fdiv_rn(1.0f, vsc);
        int8_t *kd = static_cast<int8_t *>(c.k) + kbase;
        int8_t *vd = static_cast<int8_t *>(c.v) + vbase;
#pragma unroll
        for (int cI = 0; cI < RopePairs<QK>::PPL; cI++) {
            const int i = lane + 32 * cI;
            if (i < HALF) {
                kd[i] = q8(kx.a[cI], ksc, kr);
                kd[i + HALF] = q8(kx.b[cI], ksc, kr);
            }
        }
#pragma unroll
        for (int cI = 0; cI < VPL; cI++) {
            const int i = lane + 32 * cI;
            if (i < VD) vd[i] = q8(vx[cI], vsc, vr);
        }
        if (lane == 0) {
            c.ks[row * c.n_kv + g] = ksc;
            c.vs[row * c.n_kv + g] = vsc;
        }
    } else {
        KVT *kd = static_cast<KVT *>(c.k) + kbase;
        KVT *vd = static_cast<KVT *>(c.v) + vbase;
        bool big = false;
#pragma unroll
        for (int cI = 0; cI < RopePairs<QK>::PPL; cI++) {
            const int i = lane + 32 * cI;
            if (i < HALF) {
                const KVT a = kv_from_float<KVT>(kx.a[cI]), b = kv_from_float<KVT>(kx.b[cI]);
                kd[i] = a;
                kd[i + HALF] = b;
                if constexpr (KvT<KVT>::dt == DT_BF16) {
                    uint16_t ua, ub;
                    memcpy(&ua, &a, 2);
                    memcpy(&ub, &b, 2);
                    big |= bf16x2_big(ua) || bf16x2_big(ub);
                }
            }
        }
#pragma unroll
        for (int cI = 0; cI < VPL; cI++) {
            const int i = lane + 32 * cI;
            if (i < VD) {
                const KVT x = kv_from_float<KVT>(vx[cI]);
                vd[i] = x;
                if constexpr (KvT<KVT>::dt == DT_BF16) {
                    uint16_t u;
                    memcpy(&u, &x, 2);
                    big |= bf16x2_big(u);
                }
            }
        }
        if (big && c.vbig) atomicOr(c.vbig, 1);
    }
}

// K1 kernel: one warp per (token, KV head).
template <int QK, int VD, typename KVT>
__global__ void __launch_bounds__(128) append_kernel(const AttnParams P) {
    const uint32_t lane = threadIdx.x & 31u;
    const size_t item = (size_t)blockIdx.x * 4u + (threadIdx.x >> 5);
    if (item >= (size_t)P.n_tok * P.c.n_kv) return;
    const uint32_t tok = (uint32_t)(item / P.c.n_kv), g = (uint32_t)(item % P.c.n_kv);
    const TokMeta tm = token_meta(P, tok);
    const SeqState st = P.state[tm.seq];
    const uint32_t pos = st.pos + tm.off;
    if (pos >= P.max_pos || st.n_sink >= P.c.window) {
        if (lane == 0) set_err(P.err, 2);
        return;
    }
    const uint32_t slot = kv_slot(P.c.window, st.n_sink, pos);
    const size_t row = phys_row(P.c, tm.seq, slot);
    warp_append<QK, VD, KVT>(P.c, row, g, P.k, P.v, P.act_dt,
                             ((size_t)tm.row * P.c.n_kv + g) * QK,
                             ((size_t)tm.row * P.c.n_kv + g) * VD,
                             P.rope + (size_t)pos * (QK / 2), P.knorm, (int)lane);
}

// K1 fast path: no head norm, activations already in the cache's 16-bit type,
// QK == VD. TPR = QK/8 threads per (token, KV head) row; thread t rotates the
// pairs (4t..4t+3, HALF+4t..HALF+4t+3) with 8-byte loads/stores and copies 8
// values of v with one 16-byte load/store. Same rounded statements as
// warp_norm_rope, so the rotated K is the same bits.
template <int HDIM, typename KVT>
__global__ void __launch_bounds__(256) append_vec_kernel(const AttnParams P) {
    constexpr int TPR = HDIM / 8, HALF = HDIM / 2, ROWS = 256 / TPR;
    static_assert(KvT<KVT>::dt == DT_F16 || KvT<KVT>::dt == DT_BF16, "16-bit caches");
    const int t = threadIdx.x % TPR;
    const size_t item = (size_t)blockIdx.x * ROWS + threadIdx.x / TPR;
    if (item >= (size_t)P.n_tok * P.c.n_kv) return;
    const uint32_t tok = (uint32_t)(item / P.c.n_kv), g = (uint32_t)(item % P.c.n_kv);
    const TokMeta tm = token_meta(P, tok);
    const SeqState st = P.state[tm.seq];
    const uint32_t pos = st.pos + tm.off;
    if (pos >= P.max_pos || st.n_sink >= P.c.window) {
        if (t == 0) set_err(P.err, 2);
        return;
    }
    const size_t row = phys_row(P.c, tm.seq, kv_slot(P.c.window, st.n_sink, pos));
    const size_t src = ((size_t)tm.row * P.c.n_kv + g) * HDIM;
    const KVT *k = static_cast<const KVT *>(P.k) + src;
    const KVT *v = static_cast<const KVT *>(P.v) + src;
    const uint2 ka = *reinterpret_cast<const uint2 *>(k + 4 * t);
    const uint2 kb = *reinterpret_cast<const uint2 *>(k + HALF + 4 * t);
    const uint4 vv = *reinterpret_cast<const uint4 *>(v + 8 * t);
    const float4 *cs4 = reinterpret_cast<const float4 *>(P.rope + (size_t)pos * HALF + 4 * t);
    const float4 c01 = cs4[0], c23 = cs4[1];
    const float cc[4] = {c01.x, c01.z, c23.x, c23.z}, sn[4] = {c01.y, c01.w, c23.y, c23.w};
    KVT a[4], b[4];
    memcpy(a, &ka, 8);
    memcpy(b, &kb, 8);
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const float x1 = (float)a[e], x2 = (float)b[e];
        a[e] = kv_from_float<KVT>(__fsub_rn(__fmul_rn(x1, cc[e]), __fmul_rn(x2, sn[e])));
        b[e] = kv_from_float<KVT>(__fadd_rn(__fmul_rn(x2, cc[e]), __fmul_rn(x1, sn[e])));
    }
    KVT *kd = static_cast<KVT *>(P.c.k) + row * P.c.k_dim + (size_t)g * HDIM;
    KVT *vd = static_cast<KVT *>(P.c.v) + row * P.c.v_dim + (size_t)g * HDIM;
    uint2 oa, ob;
    memcpy(&oa, a, 8);
    memcpy(&ob, b, 8);
    *reinterpret_cast<uint2 *>(kd + 4 * t) = oa;
    *reinterpret_cast<uint2 *>(kd + HALF + 4 * t) = ob;
    *reinterpret_cast<uint4 *>(vd + 8 * t) = vv;
    if constexpr (KvT<KVT>::dt == DT_BF16) {
        if (P.c.vbig && (bf16x2_big(vv.x) || bf16x2_big(vv.y) || bf16x2_big(vv.z) || bf16x2_big(vv.w) ||
                         bf16x2_big(oa.x) || bf16x2_big(oa.y) || bf16x2_big(ob.x) || bf16x2_big(ob.y)))
            atomicOr(P.c.vbig, 1);
    }
}

// ------------------------------------------------------ split-KV attention
template <int W, bool NC>
__device__ __forceinline__ void load_words(const void *p, uint32_t (&w)[W]) {
    if constexpr (W == 4) {
        if constexpr (NC) {
            asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                : "l"(p));
        } else {
            const uint4 x = *static_cast<const uint4 *>(p);
            w[0] = x.x; w[1] = x.y; w[2] = x.z; w[3] = x.w;
        }
    } else if constexpr (W == 2) {
        if constexpr (NC) {
            asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                : "=r"(w[0]), "=r"(w[1])
                : "l"(p));
        } else {
            const uint2 x = *static_cast<const uint2 *>(p);
            w[0] = x.x; w[1] = x.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < W; i++) {
            const uint32_t *q = static_cast<const uint32_t *>(p) + i;
            if constexpr (NC) asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(w[i]) : "l"(q));
            else w[i] = *q;
        }
    }
}

// I8_PERM: int8 through the ALU instead of the conversion unit. XOR with 0x80
// turns each signed byte b into b + 128; a byte permute places it in the low
// mantissa bits of 2^23 (bits 0x4B0000xx), and subtracting 2^23 + 128 leaves
// b exactly. The balanced kernel is conversion-bound on int8 rows and takes
// it; the exact-grid kernel measured slower with it and keeps the conversion.
template <typename KVT, int W, bool I8_PERM = false>
__device__ __forceinline__ void unpack(const uint32_t (&w)[W], float *f) {
#pragma unroll
    for (int i = 0; i < W; i++) {
        if constexpr (KvT<KVT>::dt == DT_I8 && I8_PERM) {
            const uint32_t x = w[i] ^ 0x80808080u;
#pragma unroll
            for (int b = 0; b < 4; b++)
                f[4 * i + b] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540u + b)) - 8388736.0f;
        } else if constexpr (KvT<KVT>::dt == DT_I8) {
            f[4 * i + 0] = (float)(int8_t)(w[i] & 0xffu);
            f[4 * i + 1] = (float)(int8_t)((w[i] >> 8) & 0xffu);
            f[4 * i + 2] = (float)(int8_t)((w[i] >> 16) & 0xffu);
            f[4 * i + 3] = (float)(int8_t)(w[i] >> 24);
        } else if constexpr (KvT<KVT>::dt == DT_F32) {
            f[i] = __uint_as_float(w[i]);
        } else if constexpr (KvT<KVT>::dt == DT_F16) {
            __half2 h;
            memcpy(&h, &w[i], 4);
            const float2 t = __half22float2(h);
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        } else {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
}

template <int QK, int VD, typename KVT, int NQ>
struct AttendShape {
    static constexpr int NW = 4;                    // warps per CTA
    static constexpr int U = 4;                     // row groups per warp iteration
    static constexpr int ES = (int)sizeof(KVT);
    static constexpr int LPR = VD * ES / 16;        // lanes per KV row (16 B of V each)
    static constexpr int RPW = 32 / LPR;            // rows per warp load
    static constexpr int EK = QK / LPR, EV = VD / LPR;
    static constexpr int WK = EK * ES / 4, WV = EV * ES / 4;
    static constexpr int ROWS_PER_ITER = NW * U * RPW;
    static_assert((VD * ES) % 16 == 0 && LPR >= 1 && LPR <= 32 && 32 % LPR == 0, "lane map");
    static_assert(QK % LPR == 0 && (EK * ES) % 4 == 0, "K chunk");
};

// Online-softmax update of one warp with UU row groups: s[u][qi] holds this
// lane's partial q.k of row group u (its EK elements), vw the loaded V words
// (I8_PERM: the int8 unpack above). Sums the partials over the row's lanes,
// applies the int8 K scale, masks rows past the item's end, then rescales and
// accumulates p V.
template <int QK, int VD, typename KVT, int NQ, int UU, bool I8_PERM = false>
__device__ __forceinline__ void consume_scores(float (&s)[UU][NQ],
                                               const uint32_t (&vw)[UU][AttendShape<QK, VD, KVT, NQ>::WV],
                                               const float (&ksc)[UU], const float (&vsc)[UU],
                                               const bool (&valid)[UU], float (&m)[NQ], float (&l)[NQ],
                                               float (&acc)[NQ][AttendShape<QK, VD, KVT, NQ>::EV]) {
    using S = AttendShape<QK, VD, KVT, NQ>;
    constexpr bool SCALED = KvT<KVT>::dt == DT_I8;
#pragma unroll
    for (int u = 0; u < UU; u++)
#pragma unroll
        for (int qi = 0; qi < NQ; qi++) {
#pragma unroll
            for (int o = S::LPR / 2; o > 0; o >>= 1)
                s[u][qi] += __shfl_xor_sync(0xffffffffu, s[u][qi], o);
            if constexpr (SCALED) s[u][qi] *= ksc[u];
            s[u][qi] = valid[u] ? s[u][qi] : -INFINITY;
        }
    float p[UU][NQ];
#pragma unroll
    for (int qi = 0; qi < NQ; qi++) {
        float t = s[0][qi];
#pragma unroll
        for (int u = 1; u < UU; u++) t = fmaxf(t, s[u][qi]);
#pragma unroll
        for (int o = S::LPR; o < 32; o <<= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
        const float mn = fmaxf(m[qi], t);
        if (mn == -INFINITY) {
#pragma unroll
            for (int u = 0; u < UU; u++) p[u][qi] = 0.0f;
            continue;
        }
        const float alpha = ex2(m[qi] - mn);
        m[qi] = mn;
        l[qi] *= alpha;
#pragma unroll
        for (int e = 0; e < S::EV; e++) acc[qi][e] *= alpha;
#pragma unroll
        for (int u = 0; u < UU; u++) {
            p[u][qi] = ex2(s[u][qi] - mn);
            l[qi] += p[u][qi];
        }
    }
#pragma unroll
    for (int u = 0; u < UU; u++) {
        float vf[S::EV];
        unpack<KVT, S::WV, I8_PERM>(vw[u], vf);
#pragma unroll
        for (int qi = 0; qi < NQ; qi++) {
            const float pv = SCALED ? p[u][qi] * vsc[u] : p[u][qi];
#pragma unroll
            for (int e = 0; e < S::EV; e++) acc[qi][e] = fmaf(pv, vf[e], acc[qi][e]);
        }
    }
}

// The same update with the partial q.k of each row group formed in f32 from
// the loaded K words.
template <int QK, int VD, typename KVT, int NQ, int UU, bool I8_PERM = false>
__device__ __forceinline__ void consume(const float (&qr)[NQ][AttendShape<QK, VD, KVT, NQ>::EK],
                                        const uint32_t (&kw)[UU][AttendShape<QK, VD, KVT, NQ>::WK],
                                        const uint32_t (&vw)[UU][AttendShape<QK, VD, KVT, NQ>::WV],
                                        const float (&ksc)[UU], const float (&vsc)[UU],
                                        const bool (&valid)[UU], float (&m)[NQ], float (&l)[NQ],
                                        float (&acc)[NQ][AttendShape<QK, VD, KVT, NQ>::EV]) {
    using S = AttendShape<QK, VD, KVT, NQ>;
    float s[UU][NQ];
#pragma unroll
    for (int u = 0; u < UU; u++) {
        float kf[S::EK];
        unpack<KVT, S::WK, I8_PERM>(kw[u], kf);
#pragma unroll
        for (int qi = 0; qi < NQ; qi++) {
            float a = 0.0f;
#pragma unroll
            for (int e = 0; e < S::EK; e++) a = fmaf(qr[qi][e], kf[e], a);
            s[u][qi] = a;
        }
    }
    consume_scores<QK, VD, KVT, NQ, UU, I8_PERM>(s, vw, ksc, vsc, valid, m, l, acc);
}

// Merge of one CTA's warps and of the splits of a (token, KV head): warps
// 0..NW-1 hold per-warp (m, l, acc) over the rows they consumed; every thread
// of the CTA calls this (the barriers are CTA-wide), threads of warps >= NW
// only take part in the barriers. With one split the CTA writes the output;
// otherwise it writes its partial and the last CTA to take a ticket merges all
// splits (nothing waits for anything).
template <int QK, int VD, typename KVT, int NQ, int NW>
__device__ __forceinline__ void attend_finish(const AttnParams &P, float (&m)[NQ], float (&l)[NQ],
                                              float (&acc)[NQ][AttendShape<QK, VD, KVT, NQ>::EV],
                                              float (*sm_o)[NQ][VD], float (*sm_m)[NQ], float (*sm_l)[NQ],
                                              int *s_last_p, uint32_t item, uint32_t split, uint32_t nsplit,
                                              uint32_t g, uint32_t out_row, int tid) {
    using S = AttendShape<QK, VD, KVT, NQ>;
    constexpr int LPR = S::LPR, EV = S::EV;
    const int lane = tid & 31, warp = tid >> 5, sub = lane % LPR, rl = lane / LPR;
    const uint32_t rep = P.rep;
    int &s_last = *s_last_p;
    // Reduce across the row lanes of the warp (m is warp-uniform).
#pragma unroll
    for (int qi = 0; qi < NQ; qi++) {
#pragma unroll
        for (int o = LPR; o < 32; o <<= 1) {
            l[qi] += __shfl_xor_sync(0xffffffffu, l[qi], o);
#pragma unroll
            for (int e = 0; e < EV; e++) acc[qi][e] += __shfl_xor_sync(0xffffffffu, acc[qi][e], o);
        }
    }
    if (warp < NW && rl == 0) {
#pragma unroll
        for (int qi = 0; qi < NQ; qi++)
#pragma unroll
            for (int e = 0; e < EV; e++) sm_o[warp][qi][sub * EV + e] = acc[qi][e];
    }
    if (warp < NW && lane == 0) {
#pragma unroll
        for (int qi = 0; qi < NQ; qi++) {
            sm_m[warp][qi] = m[qi];
            sm_l[warp][qi] = l[qi];
        }
    }
    __syncthreads();

    const size_t out_base = (size_t)out_row * P.n_heads;
    const size_t part_base = ((size_t)item * P.max_splits + split) * NQ;
    for (int idx = tid; tid < NW * 32 && idx < (int)rep * VD; idx += NW * 32) {
        const int qi = idx / VD, d = idx % VD;
        float M = sm_m[0][qi];
#pragma unroll
        for (int w = 1; w < NW; w++) M = fmaxf(M, sm_m[w][qi]);
        float o = 0.0f, L = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            const float f = ex2(sm_m[w][qi] - M);
            o += sm_o[w][qi][d] * f;
            L += sm_l[w][qi] * f;
        }
        if (nsplit == 1) {
            const uint32_t h = g * rep + qi;
            float val = o / L;
            if (P.gate) val *= 1.0f / (1.0f + ex2(-act_load(P.gate, P.act_dt, (out_base + h) * VD + d) *
                                                 1.4426950408889634f));
            out_store<VD>(P, out_row, h * VD + d, val);
        } else {
            P.part_o[(part_base + qi) * VD + d] = o;
            if (d == 0) {
                P.part_ml[(part_base + qi) * 2 + 0] = M;
                P.part_ml[(part_base + qi) * 2 + 1] = L;
            }
        }
    }
    if (nsplit == 1) return;

    // Last CTA of this (token, group) merges the splits. No CTA ever waits.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&P.counters[item], 1) == (int)nsplit - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const size_t item_base = (size_t)item * P.max_splits * NQ;
    for (int idx = tid; tid < NW * 32 && idx < (int)rep * VD; idx += NW * 32) {
        const int qi = idx / VD, d = idx % VD;
        float M = -INFINITY;
        for (uint32_t s = 0; s < nsplit; s++)
            M = fmaxf(M, __ldcg(&P.part_ml[(item_base + (size_t)s * NQ + qi) * 2]));
        float o = 0.0f, L = 0.0f;
        for (uint32_t s = 0; s < nsplit; s++) {
            const size_t b = item_base + (size_t)s * NQ + qi;
            const float f = ex2(__ldcg(&P.part_ml[b * 2]) - M);
            o += __ldcg(&P.part_o[b * VD + d]) * f;
            L += __ldcg(&P.part_ml[b * 2 + 1]) * f;
        }
        const uint32_t h = g * rep + qi;
        float val = o / L;
        if (P.gate) val *= 1.0f / (1.0f + ex2(-act_load(P.gate, P.act_dt, (out_base + h) * VD + d) *
                                             1.4426950408889634f));
        out_store<VD>(P, out_row, h * VD + d, val);
    }
    if (tid == 0) P.counters[item] = 0;
}
template <int QK, int VD, typename KVT, int NQ>
__global__ void __launch_bounds__(128) attend_kernel(const AttnParams P) {
    using S = AttendShape<QK, VD, KVT, NQ>;
    constexpr int NW = S::NW, U = S::U, LPR = S::LPR, RPW = S::RPW;
    constexpr int EK = S::EK, EV = S::EV, WK = S::WK, WV = S::WV;
    constexpr int ES = S::ES;
    constexpr bool SCALED = KvT<KVT>::dt == DT_I8;

    __shared__ float sq[NQ][QK];
    __shared__ float sm_o[NW][NQ][VD];
    __shared__ float sm_m[NW][NQ], sm_l[NW][NQ];
    __shared__ int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int sub = lane % LPR, rl = lane / LPR;
    const uint32_t n_kv = P.c.n_kv, W = P.c.window;
    uint32_t tok, g, split;
    if (P.split_cu) {
        // Exact grid: blockIdx.x enumerates the (token, split) pairs of the call.
        uint32_t lo = 0, hi = P.n_tok;
        while (hi - lo > 1) {
            const uint32_t mid = (lo + hi) >> 1;
            if (P.split_cu[mid] <= blockIdx.x) lo = mid;
            else hi = mid;
        }
        tok = lo;
        split = blockIdx.x - P.split_cu[lo];
        g = blockIdx.y;
    } else {
        tok = blockIdx.x / n_kv;
        g = blockIdx.x % n_kv;
        split = blockIdx.y;
    }
    const uint32_t item = tok * n_kv + g;
    const TokMeta tm = token_meta(P, tok);
    const SeqState st = P.state[tm.seq];
    const uint32_t pos = st.pos + tm.off, n_sink = st.n_sink;
    if (pos >= P.max_pos || n_sink >= W) {
        if (tid == 0) set_err(P.err, 2);
        return;
    }
    const Runs runs = make_runs(pos, n_sink, W);
    const uint32_t J = runs.sinks + runs.rcount;
    uint32_t nsplit, chunk;
    if (P.split_cu) {
        nsplit = P.split_cu[tok + 1] - P.split_cu[tok];
        chunk = (J + nsplit - 1) / nsplit;
    } else {
        chunk = P.chunk;
        nsplit = (J + chunk - 1) / chunk;
    }
    if (split >= nsplit) return;
    const uint32_t j0 = split * chunk;
    const uint32_t j1 = min(J, j0 + chunk);
    const bool appender = P.fuse_append && split == nsplit - 1;
    const uint32_t rep = P.rep;
    const float2 *cs = P.rope + (size_t)pos * (QK / 2);

    // q rows of this GQA group: norm + RoPE, pre-scaled into the log2 domain.
    for (int qi = warp; qi < NQ; qi += NW) {
        if (qi < (int)rep) {
            const uint32_t h = g * rep + qi;
            RopePairs<QK> x;
            warp_load_pairs<QK>(x, P.q, P.act_dt, ((size_t)tm.row * P.n_heads + h) * QK, lane);
            warp_norm_rope<QK>(x, cs, P.qnorm, lane);
#pragma unroll
            for (int c = 0; c < RopePairs<QK>::PPL; c++) {
                const int i = lane + 32 * c;
                if (i < QK / 2) {
                    sq[qi][i] = x.a[c] * P.scale_log2;
                    sq[qi][i + QK / 2] = x.b[c] * P.scale_log2;
                }
            }
        } else {
            for (int i = lane; i < QK; i += 32) sq[qi][i] = 0.0f;
        }
    }
    if (appender && warp == NW - 1) {
        const uint32_t slot = kv_slot(W, n_sink, pos);
        warp_append<QK, VD, KVT>(P.c, phys_row(P.c, tm.seq, slot), g, P.k, P.v, P.act_dt,
                                 ((size_t)tm.row * n_kv + g) * QK, ((size_t)tm.row * n_kv + g) * VD,
                                 cs, P.knorm, lane);
    }
    __syncthreads();

    float qr[NQ][EK];
#pragma unroll
    for (int qi = 0; qi < NQ; qi++)
#pragma unroll
        for (int e = 0; e < EK; e++) qr[qi][e] = sq[qi][sub * EK + e];

    float m[NQ], l[NQ], acc[NQ][EV];
#pragma unroll
    for (int qi = 0; qi < NQ; qi++) {
        m[qi] = -INFINITY;
        l[qi] = 0.0f;
#pragma unroll
        for (int e = 0; e < EV; e++) acc[qi][e] = 0.0f;
    }

    const char *kbase = static_cast<const char *>(P.c.k) + ((size_t)g * QK + (size_t)sub * EK) * ES;
    const char *vbase = static_cast<const char *>(P.c.v) + ((size_t)g * VD + (size_t)sub * EV) * ES;
    const size_t krow_bytes = (size_t)P.c.k_dim * ES, vrow_bytes = (size_t)P.c.v_dim * ES;
    const uint32_t jend = appender ? j1 - 1 : j1;

    for (uint32_t base = j0 + warp * U * RPW; base < jend; base += NW * U * RPW) {
        uint32_t kw[U][WK], vw[U][WV];
        float ksc[U], vsc[U];
        bool valid[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const uint32_t j = base + u * RPW + rl;
            valid[u] = j < jend;
            ksc[u] = vsc[u] = 0.0f;
            if (valid[u]) {
                const size_t row = phys_row(P.c, tm.seq, visit_slot(runs, j, n_sink, W));
                load_words<WK, true>(kbase + row * krow_bytes, kw[u]);
                load_words<WV, true>(vbase + row * vrow_bytes, vw[u]);
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
    if (appender && warp == NW - 1) {
        // The newest row was written by this warp above: read it back through
        // the coherent path (never the non-coherent one) after the barrier.
        uint32_t kw[1][WK], vw[1][WV];
        float ksc[1] = {0.0f}, vsc[1] = {0.0f};
        bool valid[1] = {rl == 0};
        const size_t row = phys_row(P.c, tm.seq, visit_slot(runs, J - 1, n_sink, W));
        load_words<WK, false>(kbase + row * krow_bytes, kw[0]);
        load_words<WV, false>(vbase + row * vrow_bytes, vw[0]);
        if constexpr (SCALED) {
            ksc[0] = P.c.ks[row * n_kv + g];
            vsc[0] = P.c.vs[row * n_kv + g];
        }
        consume<QK, VD, KVT, NQ, 1>(qr, kw, vw, ksc, vsc, valid, m, l, acc);
    }

    attend_finish<QK, VD, KVT, NQ, NW>(P, m, l, acc, sm_o, sm_m, sm_l, &s_last, item, split, nsplit, g, tm.row, tid);
}

}  // namespace nda
