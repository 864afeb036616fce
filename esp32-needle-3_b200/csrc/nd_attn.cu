// nd_attn.cu - host side of the C ABI declared in include/nd_attn.h.
//
// The handle plays the part of nd_model's session state and KV caches
// (engine/include/nd_model.h:129-137): a host mirror of each sequence's
// position/sink/snapshot, a device copy of the same that kernels read, the
// per-layer caches in HBM, the RoPE cos/sin table, and split-KV scratch. State
// changes reach the device through tiny kernels whose arguments are captured
// by value at launch, so they stay ordered with the attention kernels on the
// handle's stream.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/nd_attn.h"
#include "nd_async.cuh"
#include "nd_internal.h"

using nda::AttnParams;
using nda::CacheView;
using nda::SeqState;
using nda::TokMeta;

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define ND_CUDA(call)                                                                   \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                          \
            return fail(ND_ATTN_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                        __FILE__, __LINE__);                                            \
    } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

size_t dt_size(int dt) { return dt == ND_DT_I8 ? 1 : dt == ND_DT_F32 ? 4 : 2; }

struct HostSeq {
    uint32_t pos = 0, n_sink = 0, snap_pos = 0;
    int has_snap = 0;
};

// ---- small state kernels (arguments by value) ----------------------------
__global__ void set_state_kernel(SeqState *st, uint32_t seq, uint32_t pos, uint32_t n_sink) {
    st[seq].pos = pos;
    st[seq].n_sink = n_sink;
}

// Launched as a programmatic dependent: the launch after it may start at once
// (every kernel that reads positions does so after its own grid-dependency
// wait, which returns once this grid has completed), while this grid waits for
// the kernels before it, which may still read the positions, before changing
// them. So the attend launch that follows a step's advance starts under the
// previous attend launch's tail, as consecutive attend launches do.
__global__ void advance_kernel(SeqState *st, uint32_t n, const uint32_t *ids, const uint32_t *len,
                               uint32_t step) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    st[ids ? ids[i] : i].pos += len ? len[i] : step;
}

// Host-buffer decode: copies the caller's inputs from mapped host memory into
// the device buffers the attend kernels read, one unit (16, 4 or 1 bytes, as
// the segment's alignment allows) per thread so that the whole transfer is in
// flight at once: about one PCIe round trip plus the bytes at link rate. It
// lets its dependent launch start at once; that attend kernel streams K/V
// meanwhile and reads these buffers only after its grid-dependency wait, which
// returns once this grid has completed and its writes are visible.
struct IngestSeg {
    const char *src;
    char *dst;
    uint64_t units;   // of 1 << shift bytes
    uint32_t shift;
};
struct IngestParams {
    IngestSeg seg[4];
    uint64_t first[5];   // first unit of each segment, then the total
    uint32_t n;
};

__global__ void __launch_bounds__(256) ingest_kernel(const IngestParams P) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; j < P.first[P.n]; j += stride) {
        uint32_t s = 0;
        while (j >= P.first[s + 1]) s++;
        const IngestSeg g = P.seg[s];
        const uint64_t i = j - P.first[s];
        if (g.shift == 4)
            reinterpret_cast<uint4 *>(g.dst)[i] = reinterpret_cast<const uint4 *>(g.src)[i];
        else if (g.shift == 2)
            reinterpret_cast<uint32_t *>(g.dst)[i] = reinterpret_cast<const uint32_t *>(g.src)[i];
        else
            g.dst[i] = g.src[i];
    }
}

// QKV short causal convolution ahead of the path (tap_projection / tap_rows,
// nd_model.c:2361-2379, 1753-1802). One thread per (span, column) walks the
// span's tokens in order, so a history slot is never read and written by
// different threads of a launch. Column i of the token at position p is
//   0 + w[0][i]*x(p)[i] + w[1][i]*x(p-1)[i] + ...   over min(taps, p+1) taps,
// each product and sum rounded on its own, in ascending tap order; x(p-j) is
// the call's own raw row for positions inside the span, else the sequence's
// history. The raw rows of the span's last min(len, taps) positions then go
// to history slot p % taps. Columns [0, qd) are q, then k, then v.
// Launched with programmatic stream serialization: it releases its dependent
// (the attend launch) at once and waits for the kernel before it before it
// touches memory, so the attend launch of this layer may start under the
// previous layer's tail, as it does without taps.
constexpr uint32_t kTapMax = 4;
struct TapParams {
    const void *x[3];           // raw q, k, v rows of the call
    void *y[3];                 // convolved rows (same layout and type)
    uint32_t dim[3];            // qd, kd, vd
    const float *w;             // this layer's weights [q: taps][qd] [k: taps][kd] [v: taps][vd]
    float *hist;                // [max_seqs][hist_seq]
    size_t hist_seq;
    size_t hist_off[3];         // this layer's q / k / v history inside a sequence's block
    const nda::SeqSpan *spans;  // nullptr: span i = sequence i, row i, one token
    const SeqState *state;      // the span's first position is its sequence's pos
    uint32_t n_spans, taps, cols;
    int act_dt;
};

__global__ void __launch_bounds__(128) tap_kernel(const TapParams P) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // (span, column) pairs, columns fastest: a small grid (its blocks stay
    // resident beside the attend CTAs while they wait) strides over them.
    const uint64_t total = (uint64_t)P.n_spans * P.cols;
    for (uint64_t it = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; it < total;
         it += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t sp = (uint32_t)(it / P.cols), col = (uint32_t)(it % P.cols);
        const int which = col < P.dim[0] ? 0 : col < P.dim[0] + P.dim[1] ? 1 : 2;
        const uint32_t D = P.dim[which];
        const uint32_t c = col - (which > 0 ? P.dim[0] : 0u) - (which > 1 ? P.dim[1] : 0u);
        const float *w = P.w + (which > 0 ? (size_t)P.taps * P.dim[0] : 0) + (which > 1 ? (size_t)P.taps * P.dim[1] : 0);
        const nda::SeqSpan s = P.spans ? P.spans[sp] : nda::SeqSpan{sp, sp, 1u};
        const uint32_t p0 = P.state[s.seq].pos;
        float *hist = P.hist + (size_t)s.seq * P.hist_seq + P.hist_off[which];   // [taps][D]
        float wj[kTapMax], win[kTapMax];   // win[j] = x(p - 1 - j) before token p, x(p - j) after it
#pragma unroll
        for (uint32_t j = 0; j < kTapMax; j++) {
            wj[j] = j < P.taps ? w[(size_t)j * D + c] : 0.0f;
            win[j] = j + 1 < P.taps && p0 >= j + 1 ? hist[(size_t)((p0 - 1 - j) % P.taps) * D + c] : 0.0f;
        }
        for (uint32_t t = 0; t < s.len; t++) {
            const uint32_t p = p0 + t;
            const size_t xi = (size_t)(s.tok_base + t) * D + c;
            const float x = nda::act_load(P.x[which], P.act_dt, xi);
            float acc = __fadd_rn(0.0f, __fmul_rn(wj[0], x));
#pragma unroll
            for (uint32_t j = 1; j < kTapMax; j++)
                if (j < P.taps && j <= p) acc = __fadd_rn(acc, __fmul_rn(wj[j], win[j - 1]));
            nda::act_store(P.y[which], P.act_dt, xi, acc);
#pragma unroll
            for (uint32_t j = kTapMax - 1; j > 0; j--) win[j] = win[j - 1];
            win[0] = x;
        }
#pragma unroll
        for (uint32_t j = 0; j < kTapMax; j++)
            if (j < P.taps && j < s.len) hist[(size_t)((p0 + s.len - 1 - j) % P.taps) * D + c] = win[j];
    }
}

// Failure-path diagnostics: one thread waits on an mbarrier that nothing
// arrives on, for at most `limit` SM cycles, then reports the expiry through
// the status word as the hot kernels' bounded waits do (code 3).
__global__ void wait_expiry_kernel(int *err, long long limit) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    nda::mbar_init(&bar, 1);
    const long long t0 = clock64();
    while (!nda::mbar_test(&bar, 0)) {
        if (clock64() - t0 > limit) {
            nda::set_err(err, 3);
            return;
        }
    }
}

// Copies whole cache rows between a (layer-strided) cache and a dense buffer:
// dense row (l, r) <-> cache row phys_row(seq, slot0 + r) of layer l.
// `to_cache` selects the direction. Row sizes are multiples of 4 bytes.
// vbig: when copying into a bf16 K or V cache, the flag of the first layer copied
// (layer blockIdx.y's flag is vbig[blockIdx.y]); nullptr otherwise.
__global__ void rows_copy_kernel(char *cache, size_t layer_stride, char *dense, size_t dense_layer_stride,
                                 uint32_t row_words, uint32_t n_rows, CacheView c, uint32_t seq,
                                 uint32_t slot0, int to_cache, int *vbig) {
    const uint32_t l = blockIdx.y;
    bool big = false;
    for (uint32_t r = blockIdx.x; r < n_rows; r += gridDim.x) {
        const size_t pr = nda::phys_row(c, seq, slot0 + r);
        uint32_t *cw = reinterpret_cast<uint32_t *>(cache + l * layer_stride) + pr * row_words;
        uint32_t *dw = reinterpret_cast<uint32_t *>(dense + l * dense_layer_stride) + (size_t)r * row_words;
        for (uint32_t w = threadIdx.x; w < row_words; w += blockDim.x) {
            if (to_cache) {
                const uint32_t x = dw[w];
                cw[w] = x;
                big |= vbig != nullptr && nda::bf16x2_big(x);
            } else {
                dw[w] = cw[w];
            }
        }
    }
    if (big) atomicOr(vbig + l, 1);
}

}  // namespace

struct nd_attn_prefix {
    const nd_attn *owner;
    uint32_t pos, sink, live;
    size_t bytes;
    void *dev;  // image in the reference's byte order
};

struct nd_attn {
    nd_attn_config cfg;
    cudaStream_t stream = nullptr;   // where work is enqueued
    cudaStream_t own = nullptr;      // the handle's own stream
    int sm_count = 148;
    int shared_variant = 0;          // nd_attn_decode_shared kernel: 0 by call size, 1 or 2 forced (ND_ATTN_SHARED_VARIANT)
    uint32_t rep = 1, k_dim = 0, v_dim = 0, blocks_per_seq = 1, block_shift = 0;
    size_t rows_per_layer = 0, kes = 1;
    void *kc = nullptr, *vc = nullptr;
    float *ks = nullptr, *vs = nullptr;
    float2 *rope = nullptr;
    float *norms = nullptr;  // [layer][2][qk]
    std::vector<uint8_t> has_norm;
    SeqState *d_state = nullptr;
    std::vector<HostSeq> seqs;
    int32_t *d_btab = nullptr;
    float *part_o = nullptr, *part_ml = nullptr;
    float *shared_part = nullptr;    // nd_attn_decode_shared: (m, l, o) over the prefix per (token, query head)
    size_t shared_part_cap = 0;
    int *counters = nullptr;
    size_t part_slots = 0;     // (item, split) slots the scratch holds
    size_t counter_cap = 0;    // items with a ticket counter
    TokMeta *d_tok = nullptr;
    size_t tok_cap = 0;
    nda::SeqSpan *d_spans = nullptr;
    size_t spans_cap = 0;
    uint32_t *d_u32 = nullptr;
    size_t u32_cap = 0;
    uint32_t *d_lean = nullptr;        // balanced grid: [tile prefix per token | first token per CTA]
    size_t lean_cap = 0;
    std::vector<uint32_t> lean_last;   // what d_lean holds (uploads skipped when unchanged)
    int lean_occ[8] = {0};             // CTAs per SM of each (dtype, hd, nq) instantiation, 0 = not asked yet
    std::vector<uint32_t> lean_up;     // host staging of the next d_lean image
    // The plan is a function of the call's per-token {visits, sequence,
    // position} and of constants of the handle: the key of the last plan
    // built, and its shape, let calls with the same key skip the rebuild.
    std::vector<uint32_t> lean_key, lean_key_next;
    uint64_t lean_nt = 0, lean_g = 0, lean_s = 0, lean_ch = 0, lean_nu = 0;
    std::vector<CUtensorMap> lean_kmap, lean_vmap;   // per layer, built on first use
    std::vector<CUtensorMap> lean_ksmap, lean_vsmap; // int8: the layer's scale maps
    std::vector<CUtensorMap> lean_ktmap, lean_vtmap; // K / V rows in 16-row boxes (item tails)
    nda::LeanTok lean_tok;             // a small call's tokens, passed as launch parameters
    std::vector<uint8_t> lean_map_ok;
    uint32_t lean_parity = 0;          // half of counters / partials the next balanced launch uses
    // Cache rows our most recently launched kernel may write: kNoLayer (none),
    // a layer, or kAllLayers. A balanced launch may stream K/V before that
    // kernel ends only when it cannot be writing the launch's layer.
    int last_writer = -1;
    int *err_host = nullptr;  // status word: pinned host memory mapped for the kernels
    int *d_err = nullptr;     // its device address
    // QKV short causal convolution (qkv_conv_taps > 0). Tap weights per layer
    // [q: taps][qd] [k: taps][kd] [v: taps][vd]; per sequence the history of
    // raw projections [q: layers][taps][qd], then k, then v (the reference's
    // q_hist / k_hist / v_hist, slot = position % taps) and its snapshot
    // copy; the convolved rows of a call in the activation type, sized for
    // max_seqs tokens at open (grown for larger prefills).
    float *d_tapw = nullptr, *d_hist = nullptr, *d_snaphist = nullptr;
    size_t hist_seq = 0;       // floats of history per sequence
    char *d_tapio = nullptr;
    size_t tapio_cap = 0;
    nda::SeqSpan *d_tspans = nullptr;
    size_t tspans_cap = 0;
    char *hstage = nullptr;       // host-buffer calls: pinned staging, mapped for the kernels
    char *hstage_dev = nullptr;   // its device address
    size_t hstage_cap = 0;
    int *d_vbig = nullptr;    // per layer: a bf16 K or V value f16 cannot represent was stored (sticky)
    void *dio = nullptr;
    size_t dio_cap = 0;
    uint64_t launches = 0;
    // tcgen05 prefill: work list of the last call (reused when the call's
    // shape and positions repeat).
    nda::PrefillWork *d_work = nullptr;
    size_t work_cap = 0;
    std::vector<uint32_t> work_key;
    uint32_t n_work = 0;
    // Head-sharded decode over g_world ranks (nd_attn_gather_init / _attach).
    // g_buf = this rank's gather buffer, two slots of 8-byte {data, epoch}
    // words that gathered calls alternate between; g_peer[p] = rank p's
    // buffer as mapped here (own included); g_words = words per gathered row.
    uint32_t g_world = 0, g_rank = 0, g_words = 0;
    char *g_buf = nullptr;
    size_t g_slot_bytes = 0;
    char *g_peer[nda::kMaxGather] = {};
    bool g_ready = false;
    uint32_t g_epoch = 0;
    nda::GatherView gth_call{};   // in force for the attend launch of a gathered call (G = 0 otherwise)
};

namespace {

constexpr int kNoLayer = -1, kAllLayers = -2;

// Records which cache rows the kernel about to be launched may write.
inline void note_writer(nd_attn *h, int layer_or_none) { h->last_writer = layer_or_none; }

int check_seq(const nd_attn *h, uint32_t seq) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    if (seq >= h->cfg.max_seqs) return fail(ND_ATTN_ERR_RANGE, "sequence %u >= max_seqs %u", seq, h->cfg.max_seqs);
    return ND_ATTN_OK;
}

int push_state(nd_attn *h, uint32_t seq) {
    const HostSeq &s = h->seqs[seq];
    note_writer(h, kNoLayer);
    set_state_kernel<<<1, 1, 0, h->stream>>>(h->d_state, seq, s.pos, s.n_sink);
    h->launches++;
    ND_CUDA(cudaGetLastError());
    return ND_ATTN_OK;
}

CacheView layer_view(const nd_attn *h, uint32_t layer) {
    CacheView c;
    c.k = static_cast<char *>(h->kc) + layer * h->rows_per_layer * h->k_dim * h->kes;
    c.v = static_cast<char *>(h->vc) + layer * h->rows_per_layer * h->v_dim * h->kes;
    c.ks = h->ks ? h->ks + layer * h->rows_per_layer * h->cfg.n_kv_heads : nullptr;
    c.vs = h->vs ? h->vs + layer * h->rows_per_layer * h->cfg.n_kv_heads : nullptr;
    c.k_dim = h->k_dim;
    c.v_dim = h->v_dim;
    c.n_kv = h->cfg.n_kv_heads;
    c.window = h->cfg.window;
    c.btab = h->cfg.block_size ? h->d_btab : nullptr;
    c.blocks_per_seq = h->blocks_per_seq;
    c.block_shift = h->block_shift;
    c.vbig = h->cfg.kv_dtype == ND_DT_BF16 ? h->d_vbig + layer : nullptr;
    return c;
}

template <typename T>
int grow(T **p, size_t *cap, size_t need) {
    if (need <= *cap) return ND_ATTN_OK;
    size_t n = std::max(need, *cap * 2);
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(reinterpret_cast<void **>(p), n * sizeof(T)) != cudaSuccess)
        return fail(ND_ATTN_ERR_NOMEM, "device allocation of %zu bytes failed", n * sizeof(T));
    *cap = n;
    return ND_ATTN_OK;
}

// Visited positions of a token at `pos` (sink run + recent run).
uint32_t visit_count(uint32_t pos, uint32_t n_sink, uint32_t window) {
    const uint32_t sinks = std::min(n_sink, pos + 1);
    uint32_t rcount = 0;
    if (pos + 1 > n_sink) rcount = std::min(pos + 1 - n_sink, window - n_sink);
    return sinks + rcount;
}

AttnParams base_params(nd_attn *h, uint32_t layer) {
    AttnParams P;
    memset(&P, 0, sizeof(P));
    P.act_dt = h->cfg.act_dtype;
    P.out_dt = h->cfg.out_dtype;
    P.c = layer_view(h, layer);
    P.rope = h->rope;
    P.max_pos = h->cfg.max_pos;
    if (h->has_norm[layer]) {
        P.qnorm = h->norms + (size_t)layer * 2 * h->cfg.qk_head_dim;
        P.knorm = P.qnorm + h->cfg.qk_head_dim;
    }
    P.state = h->d_state;
    P.n_heads = h->cfg.n_heads;
    P.rep = h->rep;
    P.scale_log2 = 1.4426950408889634f / sqrtf((float)h->cfg.qk_head_dim);
    P.part_o = h->part_o;
    P.part_ml = h->part_ml;
    P.counters = h->counters;
    P.err = h->d_err;
    P.gth = h->gth_call;
    return P;
}

cudaError_t attend_launch(const nd_attn *h, const AttnParams &P, dim3 grid) {
    const int qk = (int)h->cfg.qk_head_dim, vd = (int)h->cfg.v_head_dim;
    const int nq = nda::nq_for_rep(h->rep);
    switch (h->cfg.kv_dtype) {
    case ND_DT_I8: return nda::attend_launch_i8(qk, vd, nq, P, grid, h->stream);
    case ND_DT_F32: return nda::attend_launch_f32(qk, vd, nq, P, grid, h->stream);
    case ND_DT_F16: return nda::attend_launch_f16(qk, vd, nq, P, grid, h->stream);
    default: return nda::attend_launch_bf16(qk, vd, nq, P, grid, h->stream);
    }
}

cudaError_t append_launch(const nd_attn *h, const AttnParams &P) {
    const int qk = (int)h->cfg.qk_head_dim, vd = (int)h->cfg.v_head_dim;
    switch (h->cfg.kv_dtype) {
    case ND_DT_I8: return nda::append_launch_i8(qk, vd, P, h->stream);
    case ND_DT_F32: return nda::append_launch_f32(qk, vd, P, h->stream);
    case ND_DT_F16: return nda::append_launch_f16(qk, vd, P, h->stream);
    default: return nda::append_launch_bf16(qk, vd, P, h->stream);
    }
}

// Chooses the split length for `items` (token, KV head) work items whose
// longest visit run is jmax and whose runs total `rows`: enough CTAs to cover
// the SMs twice over, splits that are whole loop iterations, and no more
// splits than the scratch holds.
void choose_split(const nd_attn *h, size_t items, uint32_t jmax, size_t rows, size_t counter_cap,
                  size_t part_slots, uint32_t *chunk, uint32_t *nsplit) {
    const uint32_t per_iter = (uint32_t)nda::attend_rows_per_iter(h->cfg.kv_dtype, (int)h->cfg.v_head_dim,
                                                                  nda::nq_for_rep(h->rep));
    const size_t target = (size_t)h->sm_count * 16;
    size_t c = (rows + target - 1) / target;
    c = std::max<size_t>(c, 2 * per_iter);
    c = (c + per_iter - 1) / per_iter * per_iter;
    uint32_t ns = (uint32_t)((jmax + c - 1) / c);
    if (ns > 1 && (items > counter_cap || items * ns > part_slots)) {
        const size_t cap = items > counter_cap ? 1 : part_slots / items;
        ns = (uint32_t)std::max<size_t>(1, std::min<size_t>(cap, ns));
        c = (jmax + ns - 1) / ns;
        c = (c + per_iter - 1) / per_iter * per_iter;
        ns = (uint32_t)((jmax + c - 1) / c);
    }
    if (ns < 1) ns = 1;
    *chunk = (uint32_t)c;
    *nsplit = ns;
}

// Validates the sequences of a call; fills per-call visit statistics.
int check_call(const nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const uint32_t *len) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    if (layer >= h->cfg.n_layers) return fail(ND_ATTN_ERR_RANGE, "layer %u >= n_layers %u", layer, h->cfg.n_layers);
    if (n == 0 || n > h->cfg.max_seqs) return fail(ND_ATTN_ERR_RANGE, "%u sequences (max %u)", n, h->cfg.max_seqs);
    std::vector<uint8_t> seen(seq_ids ? h->cfg.max_seqs : 0, 0);
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = seq_ids ? seq_ids[i] : i;
        if (s >= h->cfg.max_seqs) return fail(ND_ATTN_ERR_RANGE, "sequence id %u >= max_seqs", s);
        if (seq_ids) {
            if (seen[s]) return fail(ND_ATTN_ERR_ARG, "sequence id %u listed twice", s);
            seen[s] = 1;
        }
        const uint32_t l = len ? len[i] : 1;
        const uint64_t last = (uint64_t)h->seqs[s].pos + l;
        if (last > h->cfg.max_pos)
            return fail(ND_ATTN_ERR_RANGE, "sequence %u reaches position %llu >= max_pos %u", s,
                        (unsigned long long)(last - 1), h->cfg.max_pos);
    }
    return ND_ATTN_OK;
}

int upload_tok(nd_attn *h, const std::vector<TokMeta> &tok) {
    int rc = grow(&h->d_tok, &h->tok_cap, tok.size());
    if (rc) return rc;
    ND_CUDA(cudaMemcpyAsync(h->d_tok, tok.data(), tok.size() * sizeof(TokMeta), cudaMemcpyHostToDevice,
                            h->stream));
    return ND_ATTN_OK;
}

int make_map(CUtensorMap *m, bool bf16, const void *base, uint64_t inner, uint64_t rows, uint64_t stride_bytes,
             uint32_t box_rows, uint32_t box_inner, bool swizzle);
int make_map_dt(CUtensorMap *m, int dt, const void *base, uint64_t inner, uint64_t rows, uint64_t stride_bytes,
                uint32_t box_rows, uint32_t box_inner, bool swizzle);

// History block offsets of `layer` inside a sequence's [q | k | v] history.
void tap_offsets(const nd_attn *h, uint32_t layer, size_t off[3]) {
    const size_t T = h->cfg.qkv_conv_taps, L = h->cfg.n_layers;
    const size_t qd = (size_t)h->cfg.n_heads * h->cfg.qk_head_dim, kd = h->k_dim, vd = h->v_dim;
    off[0] = layer * T * qd;
    off[1] = L * T * qd + layer * T * kd;
    off[2] = L * T * (qd + kd) + layer * T * vd;
}

// Convolves the call's raw q/k/v rows into the handle's tap buffer
// (tap_kernel) and points q/k/v at the result. spans: per sequence of the
// call {sequence, first row, rows} (host); nullptr = sequence i is row i,
// one token each. `rows` = rows of the call.
int run_taps(nd_attn *h, uint32_t layer, uint32_t n_spans, const nda::SeqSpan *spans, uint32_t rows,
             const void **q, const void **k, const void **v) {
    const nd_attn_config &c = h->cfg;
    const size_t qd = (size_t)c.n_heads * c.qk_head_dim, kd = h->k_dim, vd = h->v_dim, es = dt_size(c.act_dtype);
    const size_t off1 = ((size_t)rows * qd * es + 255) / 256 * 256, off2 = off1 + ((size_t)rows * kd * es + 255) / 256 * 256;
    const size_t need = off2 + (size_t)rows * vd * es;
    int rc = grow(&h->d_tapio, &h->tapio_cap, need);
    if (rc) return rc;
    TapParams P;
    memset(&P, 0, sizeof(P));
    if (spans) {
        rc = grow(&h->d_tspans, &h->tspans_cap, n_spans);
        if (rc) return rc;
        ND_CUDA(cudaMemcpyAsync(h->d_tspans, spans, n_spans * sizeof(nda::SeqSpan), cudaMemcpyHostToDevice, h->stream));
        P.spans = h->d_tspans;
    }
    P.x[0] = *q, P.x[1] = *k, P.x[2] = *v;
    P.y[0] = h->d_tapio, P.y[1] = h->d_tapio + off1, P.y[2] = h->d_tapio + off2;
    P.dim[0] = (uint32_t)qd, P.dim[1] = (uint32_t)kd, P.dim[2] = (uint32_t)vd;
    P.taps = c.qkv_conv_taps;
    P.cols = (uint32_t)(qd + kd + vd);
    P.w = h->d_tapw + (size_t)layer * P.taps * P.cols;
    P.hist = h->d_hist;
    P.hist_seq = h->hist_seq;
    tap_offsets(h, layer, P.hist_off);
    P.state = h->d_state;
    P.n_spans = n_spans;
    P.act_dt = c.act_dtype;
    // No note_writer: the tap kernel writes no cache, but the kernel before it
    // may still be running when the attend launch after it starts.
    cudaLaunchConfig_t lc = {};
    const uint64_t pairs = (uint64_t)n_spans * P.cols;
    lc.gridDim = dim3((uint32_t)std::min<uint64_t>((pairs + 127) / 128, (uint64_t)h->sm_count * 2));
    lc.blockDim = dim3(128);
    lc.stream = h->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    ND_CUDA(cudaLaunchKernelEx(&lc, tap_kernel, P));
    h->launches++;
    *q = P.y[0], *k = P.y[1], *v = P.y[2];
    return ND_ATTN_OK;
}

// The balanced TMA-staged attend covers 16-bit caches, and int8 caches whose
// scale rows ([n_kv] floats) are a multiple of 16 bytes (n_kv % 4 == 0: the
// scales come in as TMA boxes too) with query groups of at most two rows,
// with equal head dims of 64 or 128 (GQA
// width <= 4 at 128), calls in which no position wraps the ring, and pages
// (if any) holding whole tiles (64 rows; 128 for int8, lean_rows).
bool lean_ok(const nd_attn *h, bool no_wrap) {
    const nd_attn_config &cf = h->cfg;
    const int nq = nda::nq_for_rep(h->rep);
    const bool dt_ok = cf.kv_dtype == ND_DT_F16 || cf.kv_dtype == ND_DT_BF16 ||
                       (cf.kv_dtype == ND_DT_I8 && cf.n_kv_heads % 4 == 0 && nq <= 2);
    return no_wrap && dt_ok && cf.qk_head_dim == cf.v_head_dim &&
           (cf.qk_head_dim == 64 || (cf.qk_head_dim == 128 && nq <= 4)) &&
           (cf.block_size == 0 || cf.block_size % (uint32_t)nda::lean_rows(cf.kv_dtype == ND_DT_I8) == 0) &&
           h->rows_per_layer < 0x7fffffffu;
}

// Balanced-launch tuning: share of the tiles in static units (percent), least
// tiles per dynamic unit and dynamic units a producer holds ahead, for 16-bit
// caches (64-row tiles) and int8 caches (128-row tiles). Config-2 decode swept
// over 50-90 % static, 1-3 tiles per unit, 1-2 units ahead: 16-bit caches run
// fastest at 60-65 %, 2 tiles, 2 ahead (245k tok/s against 240k at 75 %); int8
// at 85-90 %, 1 tile, 1 ahead (31.9 us per launch against 33.9 at 75 %, 1, 2).
constexpr uint64_t kLeanStaticPct16 = 65, kLeanStaticPctI8 = 85, kLeanUnitMin16 = 2, kLeanUnitMinI8 = 1;
constexpr uint32_t kLeanAhead16 = 2, kLeanAheadI8 = 1;

// Builds the balanced-launch plan of a call into h->lean_up: per token
// {first tile, tiles per item, sequence, position} and a sentinel, then per
// unit the walk state at its first tile. Uploads it when it differs from what
// the device holds and records its shape (tiles, static units and their
// size, dynamic unit size, units).
// Unit geometry of a balanced launch of nt tiles. Launches alternate between
// two halves of the tickets and of the partial scratch (two consecutive
// launches may overlap). Unit budget per half: tickets [0, NU) plus the two
// queue counters, 2 NU partial slots.
void lean_geometry(nd_attn *h, uint64_t nt, int occ) {
    const size_t cnt_half = h->counter_cap / 2, slot_half = h->part_slots / 2;
    const uint64_t budget = std::min<uint64_t>(cnt_half - 2, slot_half / 2);
    const uint64_t G = std::min<uint64_t>({nt, (uint64_t)h->sm_count * (uint64_t)occ, budget});
    const uint64_t pct = h->cfg.kv_dtype == ND_DT_I8 ? kLeanStaticPctI8 : kLeanStaticPct16;
    const uint64_t S = std::max<uint64_t>(1, nt * pct / (100 * G));
    const uint64_t dyn = nt - G * S;
    const uint64_t umin = h->cfg.kv_dtype == ND_DT_I8 ? kLeanUnitMinI8 : kLeanUnitMin16;
    uint64_t CH = std::max<uint64_t>(umin, (dyn + 4 * G - 1) / (4 * G));
    while (G + (dyn + CH - 1) / CH > budget) CH *= 2;
    h->lean_nt = nt, h->lean_g = G, h->lean_s = S, h->lean_ch = CH, h->lean_nu = G + (dyn + CH - 1) / CH;
}

int build_lean_plan(nd_attn *h, uint32_t ntok, const std::vector<uint32_t> &vis, const std::vector<uint32_t> &tok_seq,
                    const std::vector<uint32_t> &tok_pos, int fuse_append, int occ) {
    const uint32_t n_kv = h->cfg.n_kv_heads;
    const uint32_t tr = (uint32_t)nda::lean_rows(h->cfg.kv_dtype == ND_DT_I8);
    std::vector<uint32_t> &up = h->lean_up;
    up.assign((size_t)(ntok + 1) * 4, 0u);
    uint64_t nt = 0;
    for (uint32_t t = 0; t < ntok; t++) {
        const uint32_t rows = vis[t] - (fuse_append ? 1u : 0u);
        const uint32_t T = std::max<uint32_t>(1u, (rows + tr - 1) / tr);
        up[4 * t + 0] = (uint32_t)nt;
        up[4 * t + 1] = T;
        up[4 * t + 2] = tok_seq[t];
        up[4 * t + 3] = tok_pos[t];
        nt += (uint64_t)n_kv * T;
        if (nt > 0x7fffffffu) return fail(ND_ATTN_ERR_RANGE, "launch too large");
    }
    up[4 * ntok] = (uint32_t)nt;
    lean_geometry(h, nt, occ);
    const uint64_t G = h->lean_g, S = h->lean_s, CH = h->lean_ch, NU = h->lean_nu;
    const size_t ub = up.size();
    up.resize(ub + NU * 8, 0u);
    for (uint64_t u = 0, t = 0; u < NU; u++) {
        const uint64_t x0 = u < G ? u * S : G * S + (u - G) * CH;
        while (up[4 * (t + 1)] <= x0) t++;
        const uint32_t T = up[4 * t + 1], r = (uint32_t)(x0 - up[4 * t]);
        uint32_t *e = &up[ub + 8 * u];
        e[0] = (uint32_t)t, e[1] = r / T, e[2] = r % T, e[3] = T;
        e[4] = up[4 * t], e[5] = up[4 * t + 2], e[6] = up[4 * t + 3];
    }
    if (up != h->lean_last) {
        int rc = grow(&h->d_lean, &h->lean_cap, up.size());
        if (rc) return rc;
        ND_CUDA(cudaMemcpyAsync(h->d_lean, up.data(), up.size() * sizeof(uint32_t), cudaMemcpyHostToDevice,
                                h->stream));
        h->lean_last = up;
    }
    return ND_ATTN_OK;
}

// Balanced launch: item (t, g) holds T_t = max(1, ceil((vis[t] - fuse_append)
// / 64)) tiles (the newest row of a fused append is not in the TMA stream).
// G = the CTAs the GPU holds at once; the NT tiles of the call become G
// static units of S ~ 0.65 NT / G tiles (0.75 for int8 caches), then dynamic units of CH tiles (at
// most ~4 per CTA) that CTAs take as they run dry. Each unit needs two
// partial slots and one ticket; two more counters drive the unit queue.
int run_lean(nd_attn *h, uint32_t layer, uint32_t ntok, const TokMeta *d_tok, const nda::SeqSpan *d_spans,
             uint32_t n_spans, const std::vector<uint32_t> &vis, const std::vector<uint32_t> &tok_seq,
             const std::vector<uint32_t> &tok_pos, int fuse_append, const void *q, const void *k, const void *v,
             const void *gate, void *out) {
    const nd_attn_config &cf = h->cfg;
    const uint32_t hd = cf.qk_head_dim;
    const int nq = nda::nq_for_rep(h->rep);
    const bool bf16 = cf.kv_dtype == ND_DT_BF16, i8 = cf.kv_dtype == ND_DT_I8;
    auto launch = [&](const void *km, const void *vm, const void *ksm, const void *vsm, const void *ktm,
                      const void *vtm, const nda::AttnParams &P, int *occ) {
        const nda::LeanTok *tk = &h->lean_tok;
        return i8     ? nda::attend_lean_launch_i8((int)hd, nq, km, vm, ksm, vsm, ktm, vtm, tk, P, occ, h->stream)
               : bf16 ? nda::attend_lean_launch_bf16((int)hd, nq, km, vm, ksm, vsm, ktm, vtm, tk, P, occ, h->stream)
                      : nda::attend_lean_launch_f16((int)hd, nq, km, vm, ksm, vsm, ktm, vtm, tk, P, occ, h->stream);
    };
    int &occ = h->lean_occ[(bf16 ? 4 : 0) + (nq == 1 ? 0 : nq == 2 ? 1 : nq == 4 ? 2 : 3)];
    const uint32_t tr = (uint32_t)nda::lean_rows(cf.kv_dtype == ND_DT_I8);
    AttnParams P = base_params(h, layer);
    if (occ <= 0) {
        int b = 0;
        ND_CUDA(launch(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, P, &b));
        if (b <= 0) return fail(ND_ATTN_ERR_CUDA, "balanced attend kernel does not fit on an SM");
        occ = b;
    }
    nda::LeanTok &tk = h->lean_tok;
    if (ntok <= (uint32_t)nda::kLeanParamTok) {
        // A small call's token table travels as a launch parameter (the same
        // entries as build_lean_plan's): no copy between this launch and the
        // one before, which it overlaps.
        uint64_t nt = 0;
        for (uint32_t t = 0; t < ntok; t++) {
            const uint32_t rows = vis[t] - (fuse_append ? 1u : 0u);
            const uint32_t T = std::max<uint32_t>(1u, (rows + tr - 1) / tr);
            tk.tok[t] = make_uint4((uint32_t)nt, T, tok_seq[t], tok_pos[t]);
            nt += (uint64_t)cf.n_kv_heads * T;
            if (nt > 0x7fffffffu) return fail(ND_ATTN_ERR_RANGE, "launch too large");
        }
        tk.tok[ntok] = make_uint4((uint32_t)nt, 0u, 0u, 0u);
        tk.n = ntok;
        lean_geometry(h, nt, occ);
        h->lean_key.clear();   // the next large call rebuilds its plan and geometry
    } else {
        // Plan: per token {first tile, tiles per item, sequence, position} (and
        // a sentinel), then per unit the walk state at its first tile. Rebuilt
        // only when its inputs differ from the last plan's.
        tk.n = 0;
        std::vector<uint32_t> &key = h->lean_key_next;
        key.resize((size_t)ntok * 3 + 2);
        key[0] = (uint32_t)fuse_append;
        key[1] = (uint32_t)occ;
        for (uint32_t t = 0; t < ntok; t++) {
            key[2 + 3 * t] = vis[t];
            key[3 + 3 * t] = tok_seq[t];
            key[4 + 3 * t] = tok_pos[t];
        }
        if (key != h->lean_key) {
            int rc = build_lean_plan(h, ntok, vis, tok_seq, tok_pos, fuse_append, occ);
            if (rc) return rc;
            h->lean_key.swap(key);
        }
    }
    const uint64_t nt = h->lean_nt, G = h->lean_g, S = h->lean_s, CH = h->lean_ch, NU = h->lean_nu;
    const size_t cnt_half = h->counter_cap / 2, slot_half = h->part_slots / 2;
    P.lean_ahead = cf.kv_dtype == ND_DT_I8 ? kLeanAheadI8 : kLeanAhead16;
    P.lean_s = (uint32_t)S;
    P.lean_ch = (uint32_t)CH;
    P.n_units = (uint32_t)NU;
    P.work_slot = (uint32_t)(cnt_half - 2);
    const uint32_t par = h->lean_parity;
    h->lean_parity ^= 1u;
    P.counters = h->counters + par * cnt_half;
    P.part_o = h->part_o + par * slot_half * nq * hd;
    P.part_ml = h->part_ml + par * slot_half * nq * 2;
    P.early_kv = h->last_writer == kNoLayer || (h->last_writer >= 0 && h->last_writer != (int)layer);
    P.q = q; P.k = k; P.v = v; P.gate = gate; P.out = out;
    P.tok = d_tok;
    P.spans = d_spans;
    P.n_spans = n_spans;
    P.n_tok = ntok;
    P.split_cu = h->d_lean;
    P.cta_tok = h->d_lean + (size_t)(ntok + 1) * 4;
    P.n_cta = (uint32_t)G;
    P.n_tiles = (uint32_t)nt;
    P.fuse_append = fuse_append;
    if (h->lean_map_ok.size() != cf.n_layers) {
        h->lean_kmap.resize(cf.n_layers);
        h->lean_vmap.resize(cf.n_layers);
        h->lean_ksmap.resize(cf.n_layers);
        h->lean_vsmap.resize(cf.n_layers);
        h->lean_ktmap.resize(cf.n_layers);
        h->lean_vtmap.resize(cf.n_layers);
        h->lean_map_ok.assign(cf.n_layers, 0);
    }
    if (!h->lean_map_ok[layer]) {   // the layer's cache never moves: encode its maps once
        // Rows of [n_kv][hd] elements, box {hd, TR} (item tails: {hd, 16}) at x = g * hd; int8 scales
        // [n_kv] f32 per row, box {4, TR} at x = g rounded down to 4 (16 bytes). TR = lean_rows().
        const size_t es = h->kes;
        int rc = make_map_dt(&h->lean_kmap[layer], cf.kv_dtype, P.c.k, h->k_dim, h->rows_per_layer,
                             (uint64_t)h->k_dim * es, tr, hd, false);
        if (!rc) rc = make_map_dt(&h->lean_vmap[layer], cf.kv_dtype, P.c.v, h->v_dim, h->rows_per_layer,
                                  (uint64_t)h->v_dim * es, tr, hd, false);
        if (!rc) rc = make_map_dt(&h->lean_ktmap[layer], cf.kv_dtype, P.c.k, h->k_dim, h->rows_per_layer,
                                  (uint64_t)h->k_dim * es, 16, hd, false);
        if (!rc) rc = make_map_dt(&h->lean_vtmap[layer], cf.kv_dtype, P.c.v, h->v_dim, h->rows_per_layer,
                                  (uint64_t)h->v_dim * es, 16, hd, false);
        if (!rc && i8) rc = make_map_dt(&h->lean_ksmap[layer], ND_DT_F32, P.c.ks, cf.n_kv_heads, h->rows_per_layer,
                                        (uint64_t)cf.n_kv_heads * 4, tr, 4, false);
        if (!rc && i8) rc = make_map_dt(&h->lean_vsmap[layer], ND_DT_F32, P.c.vs, cf.n_kv_heads, h->rows_per_layer,
                                        (uint64_t)cf.n_kv_heads * 4, tr, 4, false);
        if (rc) return rc;
        if (!i8) h->lean_ksmap[layer] = h->lean_kmap[layer], h->lean_vsmap[layer] = h->lean_vmap[layer];  // unused
        h->lean_map_ok[layer] = 1;
    }
    note_writer(h, fuse_append ? (int)layer : kNoLayer);
    ND_CUDA(launch(&h->lean_kmap[layer], &h->lean_vmap[layer], &h->lean_ksmap[layer], &h->lean_vsmap[layer],
                   &h->lean_ktmap[layer], &h->lean_vtmap[layer], P, nullptr));
    h->launches++;
    return ND_ATTN_OK;
}

// One attend launch over `ntok` query tokens mapped by d_tok, or d_spans, or
// identity. vis[t] = visited positions of token t. The grid is exact: token t
// gets nsplit_t = ceil(vis[t] / C) splits (C sized so the call fills the GPU
// about twice over), uploaded as a prefix sum; no CTA starts without work.
// tok_seq / tok_pos (host copies of each token's sequence and position) are
// given where no position of the call wraps the ring, else null.
int run_attend(nd_attn *h, uint32_t layer, uint32_t ntok, const TokMeta *d_tok, const nda::SeqSpan *d_spans,
               uint32_t n_spans, const std::vector<uint32_t> &vis, int fuse_append, const void *q, const void *k,
               const void *v, const void *gate, void *out, const std::vector<uint32_t> *tok_seq,
               const std::vector<uint32_t> *tok_pos) {
    const uint32_t n_kv = h->cfg.n_kv_heads;
    if (tok_seq && tok_pos && lean_ok(h, true))
        return run_lean(h, layer, ntok, d_tok, d_spans, n_spans, vis, *tok_seq, *tok_pos, fuse_append, q, k, v,
                        gate, out);
    const size_t items = (size_t)ntok * n_kv;
    if (items > 0x7fffffffu) return fail(ND_ATTN_ERR_RANGE, "launch too large");
    size_t rows = 0;
    uint32_t jmax = 1;
    for (uint32_t t = 0; t < ntok; t++) {
        rows += vis[t];
        jmax = std::max(jmax, vis[t]);
    }
    const uint32_t rpi = (uint32_t)nda::attend_rows_per_iter(h->cfg.kv_dtype, (int)h->cfg.v_head_dim,
                                                             nda::nq_for_rep(h->rep));
    size_t C = std::max<size_t>((rows * n_kv + (size_t)h->sm_count * 12 - 1) / ((size_t)h->sm_count * 12),
                                (size_t)2 * rpi);
    // The scratch holds max_split partials per (token, KV head); grow C until it fits.
    uint32_t max_split = 1;
    std::vector<uint32_t> cu(ntok + 1, 0);
    for (int attempt = 0; attempt < 64; attempt++) {
        max_split = 1;
        for (uint32_t t = 0; t < ntok; t++) {
            const uint32_t ns = (uint32_t)std::max<size_t>(1, (vis[t] + C - 1) / C);
            cu[t + 1] = cu[t] + ns;
            max_split = std::max(max_split, ns);
        }
        if (max_split == 1 || (items <= h->counter_cap && items * max_split <= h->part_slots)) break;
        C *= 2;
    }
    if (max_split > 1 && (items > h->counter_cap || items * max_split > h->part_slots)) {
        max_split = 1;   // no split at all: one CTA per (token, KV head)
        for (uint32_t t = 0; t < ntok; t++) cu[t + 1] = cu[t] + 1;
    }
    if (cu[ntok] > 0x7fffffffu) return fail(ND_ATTN_ERR_RANGE, "launch too large");
    int rc = grow(&h->d_u32, &h->u32_cap, (size_t)ntok + 1);
    if (rc) return rc;
    ND_CUDA(cudaMemcpyAsync(h->d_u32, cu.data(), (ntok + 1) * sizeof(uint32_t), cudaMemcpyHostToDevice, h->stream));
    AttnParams P = base_params(h, layer);
    P.q = q; P.k = k; P.v = v; P.gate = gate; P.out = out;
    P.tok = d_tok;
    P.spans = d_spans;
    P.n_spans = n_spans;
    P.n_tok = ntok;
    P.max_splits = max_split;
    P.split_cu = h->d_u32;
    P.fuse_append = fuse_append;
    note_writer(h, fuse_append ? (int)layer : kNoLayer);
    ND_CUDA(attend_launch(h, P, dim3(cu[ntok], n_kv, 1)));
    h->launches++;
    (void)jmax;
    return ND_ATTN_OK;
}

size_t act_bytes(const nd_attn *h, size_t tokens, int which) {
    const nd_attn_config &c = h->cfg;
    const size_t a = dt_size(c.act_dtype);
    switch (which) {
    case 0: return tokens * c.n_heads * c.qk_head_dim * a;          // q
    case 1: return tokens * c.n_kv_heads * c.qk_head_dim * a;       // k
    case 2: return tokens * c.n_kv_heads * c.v_head_dim * a;        // v
    case 3: return tokens * c.n_heads * c.v_head_dim * a;           // gate
    default: return tokens * c.n_heads * c.v_head_dim * dt_size(c.out_dtype);  // out
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2D map over rows of `inner` 16-bit elements (row stride `stride_bytes`), box
// 64 elements x box_rows rows, 128-byte swizzle, out-of-range rows read as zero.
// 2D tensor map of `dt` elements (ND_DT_*): rows of `inner` elements,
// `stride_bytes` apart; box `box_inner` x `box_rows`.
int make_map_dt(CUtensorMap *m, int dt, const void *base, uint64_t inner, uint64_t rows, uint64_t stride_bytes,
                uint32_t box_rows, uint32_t box_inner, bool swizzle) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return fail(ND_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType t = dt == ND_DT_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                  : dt == ND_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                  : dt == ND_DT_I8  ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const CUresult r = fn(m, t, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ND_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return ND_ATTN_OK;
}
// The RoPE table (hd 64: 32 (cos, sin) pairs = 256 B per position) as a 3D
// map [max_pos][2 halves][32 floats] with the 128-byte swizzle, box 32 x 2 x
// 128: one prefill tile's 128 consecutive positions.
int make_rope_map(CUtensorMap *m, const void *rope, uint32_t max_pos) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return fail(ND_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[3] = {32, 2, max_pos};
    const cuuint64_t strides[2] = {128, 256};
    const cuuint32_t box[3] = {32, 2, 128};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void *>(rope), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ND_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled (rope) failed (%d)", (int)r);
    return ND_ATTN_OK;
}
int make_map(CUtensorMap *m, bool bf16, const void *base, uint64_t inner, uint64_t rows, uint64_t stride_bytes,
             uint32_t box_rows, uint32_t box_inner, bool swizzle) {
    return make_map_dt(m, bf16 ? ND_DT_BF16 : ND_DT_F16, base, inner, rows, stride_bytes, box_rows, box_inner,
                       swizzle);
}

// The tensor-core prefill serves 16-bit caches of head dim 64 in the
// contiguous layout, with q in the cache's element type and 16-byte aligned.
bool tc_prefill_ok(const nd_attn *h, const void *q) {
    const nd_attn_config &c = h->cfg;
    return (c.kv_dtype == ND_DT_BF16 || c.kv_dtype == ND_DT_F16) && c.act_dtype == c.kv_dtype &&
           c.qk_head_dim == 64 && c.v_head_dim == 64 && (c.block_size == 0 || c.block_size % 64 == 0) &&
           (reinterpret_cast<uintptr_t>(q) & 15u) == 0;
}

int run_prefill_tc(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const uint32_t *len,
                   const std::vector<uint32_t> &cu, size_t total, const void *q, const void *gate, void *out) {
    const nd_attn_config &c = h->cfg;
    // Work list: (sequence, query head, 128-token tile), longest KV run first.
    std::vector<uint32_t> key;
    key.reserve(3 * n + 2);
    key.push_back(n);
    key.push_back(c.n_heads);
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = seq_ids ? seq_ids[i] : i;
        key.push_back(s);
        key.push_back(len[i]);
        key.push_back(h->seqs[s].pos);
    }
    if (key != h->work_key) {
        std::vector<std::vector<nda::PrefillWork>> by_tiles;
        size_t count = 0;
        for (uint32_t i = 0; i < n; i++) {
            const uint32_t s = seq_ids ? seq_ids[i] : i, pos0 = h->seqs[s].pos;
            for (uint32_t t0 = 0; t0 < len[i]; t0 += 128) {
                const uint32_t rows = std::min(128u, len[i] - t0);
                const uint32_t nkv = (pos0 + t0 + rows + 63) / 64;   // 64-key tiles the item reads
                if (by_tiles.size() <= nkv) by_tiles.resize(nkv + 1);
                for (uint32_t hq = 0; hq < c.n_heads; hq++)
                    by_tiles[nkv].push_back(nda::PrefillWork{s, cu[i], t0, rows, hq, pos0});
                count += c.n_heads;
            }
        }
        if (count > 0x7fffffffu) return fail(ND_ATTN_ERR_RANGE, "prefill too large");
        std::vector<nda::PrefillWork> work;
        work.reserve(count);
        for (size_t t = by_tiles.size(); t-- > 0;) work.insert(work.end(), by_tiles[t].begin(), by_tiles[t].end());
        int rc = grow(&h->d_work, &h->work_cap, work.size());
        if (rc) return rc;
        ND_CUDA(cudaMemcpyAsync(h->d_work, work.data(), work.size() * sizeof(nda::PrefillWork),
                                cudaMemcpyHostToDevice, h->stream));
        h->work_key = key;
        h->n_work = (uint32_t)work.size();
    }
    const bool bf16 = c.kv_dtype == ND_DT_BF16;
    CUtensorMap qm, km, vm;
    CacheView cv = layer_view(h, layer);
    int rc = make_map(&qm, bf16, q, (uint64_t)c.n_heads * 64, total, (uint64_t)c.n_heads * 64 * 2, 128, 64, true);
    if (!rc) rc = make_map(&km, bf16, cv.k, h->k_dim, h->rows_per_layer, (uint64_t)h->k_dim * 2, 64, 64, true);
    if (!rc) rc = make_map(&vm, bf16, cv.v, h->v_dim, h->rows_per_layer, (uint64_t)h->v_dim * 2, 64, 64, true);
    // Output (and gate) tiles go through shared memory and TMA: 128 rows x 64
    // elements of one head, 128-byte swizzle (f32 out: two 32-element boxes).
    CUtensorMap om, csm;
    const bool o32 = c.out_dtype == ND_DT_F32;
    const uint64_t ocols = (uint64_t)c.n_heads * 64;
    if (!rc) rc = make_map_dt(&om, c.out_dtype, out, ocols, total, ocols * (o32 ? 4 : 2), 128, o32 ? 32 : 64, true);
    if (!rc) rc = make_rope_map(&csm, h->rope, c.max_pos);
    if (rc) return rc;
    nda::PrefillTcParams P;
    P.work = h->d_work;
    P.n_work = h->n_work;
    P.rope = h->rope;
    P.qnorm = h->has_norm[layer] ? h->norms + (size_t)layer * 2 * c.qk_head_dim : nullptr;
    P.gate = gate;
    P.out = out;
    P.act_dt = c.act_dtype;
    P.out_dt = c.out_dtype;
    P.n_heads = c.n_heads;
    P.rep = h->rep;
    P.window = c.window;
    P.btab = cv.btab;
    P.vbig = cv.vbig;
    P.blocks_per_seq = cv.blocks_per_seq;
    P.block_shift = cv.block_shift;
    P.scale_log2 = 1.4426950408889634f / sqrtf((float)c.qk_head_dim);
    P.err = h->d_err;
    note_writer(h, kNoLayer);
    const uint32_t grid = std::min<uint32_t>(h->n_work, 2u * (uint32_t)h->sm_count);   // persistent, 2 per SM
    ND_CUDA(nda::prefill_tc_launch(bf16, &qm, &km, &vm, &om, &csm, P, grid, h->stream));
    h->launches += bf16 ? 2 : 1;
    return ND_ATTN_OK;
}

}  // namespace

int nda::attend_rows_per_iter(int kv_dt, int vd, int nq) {
    const int es = kv_dt == ND_DT_I8 ? 1 : kv_dt == ND_DT_F32 ? 4 : 2;
    const int lpr = vd * es / 16;
    return 4 * 4 * (32 / lpr) + 0 * nq;   // warps x row groups x rows per warp load
}

// ============================================================ C ABI
extern "C" {

void nd_attn_config_init(nd_attn_config *cfg) {
    if (!cfg) return;
    memset(cfg, 0, sizeof(*cfg));
    cfg->n_layers = 1;
    cfg->n_heads = 8;
    cfg->n_kv_heads = 8;
    cfg->qk_head_dim = 64;
    cfg->v_head_dim = 64;
    cfg->window = 384;
    cfg->max_seqs = 1;
    cfg->rope_theta = 10000.0f;
    cfg->kv_dtype = ND_DT_F32;
    cfg->act_dtype = ND_DT_F32;
    cfg->out_dtype = ND_DT_F32;
}

int nd_attn_open(const nd_attn_config *cfg_in, nd_attn **out) {
    if (!cfg_in || !out) return fail(ND_ATTN_ERR_ARG, "null argument");
    *out = nullptr;
    nd_attn_config cfg = *cfg_in;
    if (cfg.max_pos == 0) cfg.max_pos = cfg.window;
    if (!nda::head_dims_supported(cfg.qk_head_dim, cfg.v_head_dim))
        return fail(ND_ATTN_ERR_GEOM, "head dims (%u,%u) not compiled", cfg.qk_head_dim, cfg.v_head_dim);
    if (cfg.n_kv_heads == 0 || cfg.n_heads % cfg.n_kv_heads || cfg.n_heads / cfg.n_kv_heads > 8)
        return fail(ND_ATTN_ERR_GEOM, "heads %u/%u: need n_heads %% n_kv_heads == 0 and ratio <= 8",
                    cfg.n_heads, cfg.n_kv_heads);
    if (cfg.n_layers == 0 || cfg.window < 1 || cfg.max_seqs == 0)
        return fail(ND_ATTN_ERR_GEOM, "n_layers, window and max_seqs must be positive");
    if (cfg.kv_dtype < ND_DT_I8 || cfg.kv_dtype > ND_DT_BF16 || cfg.act_dtype < ND_DT_F32 ||
        cfg.act_dtype > ND_DT_BF16 || cfg.out_dtype < ND_DT_F32 || cfg.out_dtype > ND_DT_BF16)
        return fail(ND_ATTN_ERR_ARG, "bad dtype");
    if (cfg.qkv_conv_taps > kTapMax) return fail(ND_ATTN_ERR_GEOM, "qkv_conv_taps %u > %u", cfg.qkv_conv_taps, kTapMax);
    if (cfg.block_size) {
        if (cfg.block_size & (cfg.block_size - 1)) return fail(ND_ATTN_ERR_GEOM, "block_size must be a power of two");
        if (cfg.window % cfg.block_size) return fail(ND_ATTN_ERR_GEOM, "window must be a multiple of block_size");
        if (cfg.n_blocks == 0) cfg.n_blocks = (uint32_t)((size_t)cfg.max_seqs * cfg.window / cfg.block_size);
    }

    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(ND_ATTN_ERR_NOGPU, "no CUDA device");
    if (cfg.device < 0 || cfg.device >= ndev) return fail(ND_ATTN_ERR_ARG, "device %d of %d", cfg.device, ndev);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, cfg.device) != cudaSuccess || prop.major != 10)
        return fail(ND_ATTN_ERR_NOGPU, "device %d is not sm_100 (the library is built for sm_100a only)", cfg.device);
    DeviceGuard dg(cfg.device);

    nd_attn *h = new nd_attn();
    h->cfg = cfg;
    h->sm_count = prop.multiProcessorCount;
    // ND_ATTN_SHARED_VARIANT=1 or 2 makes nd_attn_decode_shared use that
    // kernel whatever the call's size (variant 2 where it is built), so tests
    // cover both on small calls.
    if (const char *sv = getenv("ND_ATTN_SHARED_VARIANT")) {
        const int x = atoi(sv);
        h->shared_variant = x == 1 || x == 2 ? x : 0;
    }
    h->rep = cfg.n_heads / cfg.n_kv_heads;
    h->k_dim = cfg.n_kv_heads * cfg.qk_head_dim;
    h->v_dim = cfg.n_kv_heads * cfg.v_head_dim;
    h->kes = dt_size(cfg.kv_dtype);
    if (cfg.block_size) {
        h->blocks_per_seq = cfg.window / cfg.block_size;
        while ((1u << h->block_shift) < cfg.block_size) h->block_shift++;
        h->rows_per_layer = (size_t)cfg.n_blocks * cfg.block_size;
    } else {
        h->rows_per_layer = (size_t)cfg.max_seqs * cfg.window;
    }
    h->seqs.assign(cfg.max_seqs, HostSeq());
    h->has_norm.assign(cfg.n_layers, 0);

    auto bail = [&](int code) {
        nd_attn_close(h);
        return code;
    };
    if (cudaStreamCreateWithFlags(&h->own, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(ND_ATTN_ERR_CUDA, "stream creation failed"));
    h->stream = h->own;
    const size_t kbytes = cfg.n_layers * h->rows_per_layer * h->k_dim * h->kes;
    const size_t vbytes = cfg.n_layers * h->rows_per_layer * h->v_dim * h->kes;
    if (cudaMalloc(&h->kc, kbytes) != cudaSuccess || cudaMalloc(&h->vc, vbytes) != cudaSuccess)
        return bail(fail(ND_ATTN_ERR_NOMEM, "KV cache allocation (%zu + %zu bytes) failed", kbytes, vbytes));
    cudaMemsetAsync(h->kc, 0, kbytes, h->stream);
    cudaMemsetAsync(h->vc, 0, vbytes, h->stream);
    if (cfg.kv_dtype == ND_DT_I8) {
        const size_t sb = cfg.n_layers * h->rows_per_layer * cfg.n_kv_heads * sizeof(float);
        if (cudaMalloc(&h->ks, sb) != cudaSuccess || cudaMalloc(&h->vs, sb) != cudaSuccess)
            return bail(fail(ND_ATTN_ERR_NOMEM, "scale allocation failed"));
        cudaMemsetAsync(h->ks, 0, sb, h->stream);
        cudaMemsetAsync(h->vs, 0, sb, h->stream);
    }
    // RoPE table with the reference's own expressions (nd_model.c:1233-1236,
    // 2949-2954), so the rotated K is bit-identical to the host engine's.
    {
        const uint32_t half = cfg.qk_head_dim / 2;
        std::vector<float> inv(half);
        for (uint32_t i = 0; i < half; i++)
            inv[i] = 1.0f / powf(cfg.rope_theta, (float)(2 * i) / (float)cfg.qk_head_dim);
        std::vector<float2> tab((size_t)cfg.max_pos * half);
        for (uint32_t p = 0; p < cfg.max_pos; p++)
            for (uint32_t i = 0; i < half; i++) {
                const float angle = (float)p * inv[i];
                tab[(size_t)p * half + i] = make_float2(cosf(angle), sinf(angle));
            }
        if (cudaMalloc(&h->rope, tab.size() * sizeof(float2)) != cudaSuccess)
            return bail(fail(ND_ATTN_ERR_NOMEM, "rope table allocation failed"));
        if (cudaMemcpy(h->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(ND_ATTN_ERR_CUDA, "rope table upload failed"));
    }
    if (cudaMalloc(&h->norms, (size_t)cfg.n_layers * 2 * cfg.qk_head_dim * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&h->d_state, cfg.max_seqs * sizeof(SeqState)) != cudaSuccess ||
        cudaMalloc(&h->d_vbig, cfg.n_layers * sizeof(int)) != cudaSuccess ||
        cudaHostAlloc(reinterpret_cast<void **>(&h->err_host), sizeof(int),
                      cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void **>(&h->d_err), h->err_host, 0) != cudaSuccess)
        return bail(fail(ND_ATTN_ERR_NOMEM, "state allocation failed"));
    *h->err_host = 0;
    cudaMemsetAsync(h->d_state, 0, cfg.max_seqs * sizeof(SeqState), h->stream);
    // The small kernels between attend launches ask for the shared-memory
    // carveout the attend kernels need, so an SM that ran one need not be
    // reconfigured before it takes an attend CTA.
    cudaFuncSetAttribute(ingest_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    cudaFuncSetAttribute(advance_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    cudaMemsetAsync(h->d_vbig, 0, cfg.n_layers * sizeof(int), h->stream);
    if (cfg.block_size) {
        const size_t nb = (size_t)cfg.max_seqs * h->blocks_per_seq;
        std::vector<int32_t> ident(nb);
        for (size_t i = 0; i < nb; i++) ident[i] = (int32_t)(i % cfg.n_blocks);
        if (cudaMalloc(&h->d_btab, nb * sizeof(int32_t)) != cudaSuccess)
            return bail(fail(ND_ATTN_ERR_NOMEM, "block table allocation failed"));
        if (cudaMemcpy(h->d_btab, ident.data(), nb * sizeof(int32_t), cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(ND_ATTN_ERR_CUDA, "block table upload failed"));
    }
    // Split-KV scratch: up to 64 MB of partial outputs, tickets for every
    // (sequence, KV head) of a full decode.
    {
        const size_t nq = (size_t)nda::nq_for_rep(h->rep);
        const size_t per_slot = nq * (cfg.v_head_dim + 2) * sizeof(float);
        // Tickets for every (sequence, KV head) of a full decode, and, in each
        // of two halves, for every unit of a balanced launch (at most 5 per
        // CTA, 16 CTAs per SM).
        h->counter_cap = std::max<size_t>((size_t)cfg.max_seqs * cfg.n_kv_heads, (size_t)h->sm_count * 160);
        h->part_slots = std::max<size_t>(h->counter_cap * 4, (64ull << 20) / per_slot);
        if (cudaMalloc(&h->part_o, h->part_slots * nq * cfg.v_head_dim * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&h->part_ml, h->part_slots * nq * 2 * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&h->counters, h->counter_cap * sizeof(int)) != cudaSuccess)
            return bail(fail(ND_ATTN_ERR_NOMEM, "split-KV scratch allocation failed"));
        cudaMemsetAsync(h->counters, 0, h->counter_cap * sizeof(int), h->stream);
    }
    if (cfg.qkv_conv_taps) {
        // Identity taps until set (w[0] = 1), zero history; the tap buffer
        // serves a decode of every sequence without growing.
        const size_t T = cfg.qkv_conv_taps, qd = (size_t)cfg.n_heads * cfg.qk_head_dim;
        const size_t D = qd + h->k_dim + h->v_dim;
        h->hist_seq = (size_t)cfg.n_layers * T * D;
        std::vector<float> w((size_t)cfg.n_layers * T * D, 0.0f);
        for (size_t l = 0; l < cfg.n_layers; l++) {
            float *wl = w.data() + l * T * D;
            for (size_t i = 0; i < qd; i++) wl[i] = 1.0f;
            for (size_t i = 0; i < h->k_dim; i++) wl[T * qd + i] = 1.0f;
            for (size_t i = 0; i < h->v_dim; i++) wl[T * (qd + h->k_dim) + i] = 1.0f;
        }
        const size_t es = dt_size(cfg.act_dtype), m = cfg.max_seqs;
        if (cudaMalloc(&h->d_tapw, w.size() * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&h->d_hist, m * h->hist_seq * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&h->d_snaphist, m * h->hist_seq * sizeof(float)) != cudaSuccess ||
            grow(&h->d_tapio, &h->tapio_cap, (m * qd * es + 255) / 256 * 256 + (m * h->k_dim * es + 255) / 256 * 256 +
                                                m * h->v_dim * es) != ND_ATTN_OK)
            return bail(fail(ND_ATTN_ERR_NOMEM, "conv tap state allocation failed"));
        if (cudaMemcpy(h->d_tapw, w.data(), w.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(ND_ATTN_ERR_CUDA, "conv tap upload failed"));
        cudaMemsetAsync(h->d_hist, 0, m * h->hist_seq * sizeof(float), h->stream);
        cudaMemsetAsync(h->d_snaphist, 0, m * h->hist_seq * sizeof(float), h->stream);
    }
    if (cudaStreamSynchronize(h->stream) != cudaSuccess)
        return bail(fail(ND_ATTN_ERR_CUDA, "initialisation failed: %s", cudaGetErrorString(cudaGetLastError())));
    *out = h;
    return ND_ATTN_OK;
}

void nd_attn_close(nd_attn *h) {
    if (!h) return;
    DeviceGuard dg(h->cfg.device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    cudaFree(h->kc); cudaFree(h->vc); cudaFree(h->ks); cudaFree(h->vs);
    cudaFree(h->rope); cudaFree(h->norms); cudaFree(h->d_state); cudaFree(h->d_btab);
    cudaFree(h->part_o); cudaFree(h->part_ml); cudaFree(h->counters); cudaFree(h->shared_part);
    cudaFree(h->d_tok); cudaFree(h->d_u32); cudaFree(h->d_lean); cudaFree(h->d_vbig); cudaFree(h->dio); cudaFree(h->d_work); cudaFree(h->d_spans);
    cudaFree(h->d_tapw); cudaFree(h->d_hist); cudaFree(h->d_snaphist); cudaFree(h->d_tapio); cudaFree(h->d_tspans);
    if (h->hstage) cudaFreeHost(h->hstage);
    if (h->err_host) cudaFreeHost(h->err_host);
    if (h->own) cudaStreamDestroy(h->own);
    for (uint32_t p = 0; p < h->g_world; p++)
        if (h->g_peer[p] && h->g_peer[p] != h->g_buf) cudaIpcCloseMemHandle(h->g_peer[p]);
    cudaFree(h->g_buf);
    delete h;
}

int nd_attn_set_head_norm(nd_attn *h, uint32_t layer, const float *q_scale, const float *k_scale) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    if (layer >= h->cfg.n_layers) return fail(ND_ATTN_ERR_RANGE, "layer %u", layer);
    if (!q_scale != !k_scale) return fail(ND_ATTN_ERR_ARG, "q and k norm scales go together");
    DeviceGuard dg(h->cfg.device);
    if (!q_scale) {
        h->has_norm[layer] = 0;
        return ND_ATTN_OK;
    }
    const size_t qk = h->cfg.qk_head_dim;
    ND_CUDA(cudaStreamSynchronize(h->stream));
    ND_CUDA(cudaMemcpy(h->norms + layer * 2 * qk, q_scale, qk * sizeof(float), cudaMemcpyHostToDevice));
    ND_CUDA(cudaMemcpy(h->norms + layer * 2 * qk + qk, k_scale, qk * sizeof(float), cudaMemcpyHostToDevice));
    h->has_norm[layer] = 1;
    return ND_ATTN_OK;
}

int nd_attn_set_conv_taps(nd_attn *h, uint32_t layer, const float *wq, const float *wk, const float *wv) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    if (!h->cfg.qkv_conv_taps) return fail(ND_ATTN_ERR_ARG, "the handle was opened without conv taps");
    if (layer >= h->cfg.n_layers) return fail(ND_ATTN_ERR_RANGE, "layer %u", layer);
    if (!wq || !wk || !wv) return fail(ND_ATTN_ERR_ARG, "null tap weights");
    DeviceGuard dg(h->cfg.device);
    const size_t T = h->cfg.qkv_conv_taps, qd = (size_t)h->cfg.n_heads * h->cfg.qk_head_dim;
    float *wl = h->d_tapw + (size_t)layer * T * (qd + h->k_dim + h->v_dim);
    ND_CUDA(cudaStreamSynchronize(h->stream));
    ND_CUDA(cudaMemcpy(wl, wq, T * qd * sizeof(float), cudaMemcpyHostToDevice));
    ND_CUDA(cudaMemcpy(wl + T * qd, wk, T * h->k_dim * sizeof(float), cudaMemcpyHostToDevice));
    ND_CUDA(cudaMemcpy(wl + T * (qd + h->k_dim), wv, T * h->v_dim * sizeof(float), cudaMemcpyHostToDevice));
    return ND_ATTN_OK;
}

// Tap history of a sequence: cleared by reset (nd_model.c:1575-1580), copied
// by snapshot and rewind (1423-1425, 1451-1453).
static int hist_reset(nd_attn *h, uint32_t seq) {
    if (!h->cfg.qkv_conv_taps) return ND_ATTN_OK;
    ND_CUDA(cudaMemsetAsync(h->d_hist + seq * h->hist_seq, 0, h->hist_seq * sizeof(float), h->stream));
    return ND_ATTN_OK;
}
static int hist_copy(nd_attn *h, uint32_t seq, bool to_snapshot) {
    if (!h->cfg.qkv_conv_taps) return ND_ATTN_OK;
    float *live = h->d_hist + seq * h->hist_seq, *snap = h->d_snaphist + seq * h->hist_seq;
    ND_CUDA(cudaMemcpyAsync(to_snapshot ? snap : live, to_snapshot ? live : snap, h->hist_seq * sizeof(float),
                            cudaMemcpyDeviceToDevice, h->stream));
    return ND_ATTN_OK;
}

int nd_attn_reset(nd_attn *h, uint32_t seq) {
    int rc = check_seq(h, seq);
    if (rc) return rc;
    DeviceGuard dg(h->cfg.device);
    h->seqs[seq] = HostSeq();
    rc = hist_reset(h, seq);
    return rc ? rc : push_state(h, seq);
}

int nd_attn_set_sink(nd_attn *h, uint32_t seq, uint32_t n) {
    int rc = check_seq(h, seq);
    if (rc) return rc;
    DeviceGuard dg(h->cfg.device);
    const uint32_t cap = h->cfg.window > 64u ? h->cfg.window - 64u : 0u;  // ND_MIN_RECENT
    h->seqs[seq].n_sink = n > cap ? cap : n;
    return push_state(h, seq);
}

int nd_attn_snapshot(nd_attn *h, uint32_t seq) {
    int rc = check_seq(h, seq);
    if (rc) return rc;
    HostSeq &s = h->seqs[seq];
    const uint32_t cap = h->cfg.window > 64u ? h->cfg.window - 64u : 0u;
    DeviceGuard dg(h->cfg.device);
    s.n_sink = s.pos > cap ? cap : s.pos;
    s.snap_pos = s.pos;
    s.has_snap = 1;
    rc = hist_copy(h, seq, true);
    return rc ? rc : push_state(h, seq);
}

int nd_attn_rewind(nd_attn *h, uint32_t seq) {
    int rc = check_seq(h, seq);
    if (rc) return rc;
    HostSeq &s = h->seqs[seq];
    if (!s.has_snap) return nd_attn_reset(h, seq);
    DeviceGuard dg(h->cfg.device);
    s.pos = s.snap_pos;
    rc = hist_copy(h, seq, false);
    return rc ? rc : push_state(h, seq);
}

int nd_attn_advance(nd_attn *h, uint32_t n, const uint32_t *seq_ids, const uint32_t *len) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    if (n == 0) return ND_ATTN_OK;
    if (n > h->cfg.max_seqs) return fail(ND_ATTN_ERR_RANGE, "%u sequences", n);
    for (uint32_t i = 0; i < n; i++)
        if ((seq_ids ? seq_ids[i] : i) >= h->cfg.max_seqs) return fail(ND_ATTN_ERR_RANGE, "sequence id");
    DeviceGuard dg(h->cfg.device);
    const uint32_t *d_ids = nullptr, *d_len = nullptr;
    if (seq_ids || len) {
        int rc = grow(&h->d_u32, &h->u32_cap, 2 * (size_t)n);
        if (rc) return rc;
        if (seq_ids) {
            ND_CUDA(cudaMemcpyAsync(h->d_u32, seq_ids, n * sizeof(uint32_t), cudaMemcpyHostToDevice, h->stream));
            d_ids = h->d_u32;
        }
        if (len) {
            ND_CUDA(cudaMemcpyAsync(h->d_u32 + n, len, n * sizeof(uint32_t), cudaMemcpyHostToDevice, h->stream));
            d_len = h->d_u32 + n;
        }
    }
    for (uint32_t i = 0; i < n; i++) h->seqs[seq_ids ? seq_ids[i] : i].pos += len ? len[i] : 1;
    // No note_writer: the advance writes no cache, but the kernel before it may
    // still be running when the attend launch after it starts.
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((n + 127) / 128);
    lc.blockDim = dim3(128);
    lc.stream = h->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    ND_CUDA(cudaLaunchKernelEx(&lc, advance_kernel, h->d_state, n, d_ids, d_len, 1u));
    h->launches++;
    ND_CUDA(cudaGetLastError());
    return ND_ATTN_OK;
}

int nd_attn_get_state(nd_attn *h, uint32_t seq, uint32_t *pos, uint32_t *n_sink) {
    int rc = check_seq(h, seq);
    if (rc) return rc;
    if (pos) *pos = h->seqs[seq].pos;
    if (n_sink) *n_sink = h->seqs[seq].n_sink;
    return ND_ATTN_OK;
}

int nd_attn_set_state(nd_attn *h, uint32_t seq, uint32_t pos, uint32_t n_sink) {
    int rc = check_seq(h, seq);
    if (rc) return rc;
    if (n_sink >= h->cfg.window) return fail(ND_ATTN_ERR_RANGE, "n_sink %u >= window", n_sink);
    DeviceGuard dg(h->cfg.device);
    h->seqs[seq].pos = pos;
    h->seqs[seq].n_sink = n_sink;
    return push_state(h, seq);
}

int nd_attn_decode(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const void *q,
                   const void *k, const void *v, const void *gate, void *out) {
    int rc = check_call(h, layer, n, seq_ids, nullptr);
    if (rc) return rc;
    if (!q || !k || !v || !out) return fail(ND_ATTN_ERR_ARG, "null tensor");
    DeviceGuard dg(h->cfg.device);
    if (h->cfg.qkv_conv_taps) {
        std::vector<nda::SeqSpan> sp;
        if (seq_ids) {
            sp.resize(n);
            for (uint32_t i = 0; i < n; i++) sp[i] = nda::SeqSpan{seq_ids[i], i, 1u};
        }
        rc = run_taps(h, layer, n, seq_ids ? sp.data() : nullptr, n, &q, &k, &v);
        if (rc) return rc;
    }
    std::vector<uint32_t> vis(n), tseq(n), tpos(n);
    bool no_wrap = true;
    for (uint32_t i = 0; i < n; i++) {
        tseq[i] = seq_ids ? seq_ids[i] : i;
        const HostSeq &s = h->seqs[tseq[i]];
        vis[i] = visit_count(s.pos, s.n_sink, h->cfg.window);
        tpos[i] = s.pos;
        no_wrap = no_wrap && s.pos < h->cfg.window;
    }
    const TokMeta *d_tok = nullptr;
    if (seq_ids) {
        std::vector<TokMeta> tok(n);
        for (uint32_t i = 0; i < n; i++) tok[i] = TokMeta{seq_ids[i], 0u, i};
        rc = upload_tok(h, tok);
        if (rc) return rc;
        d_tok = h->d_tok;
    }
    return run_attend(h, layer, n, d_tok, nullptr, 0, vis, 1, q, k, v, gate, out, no_wrap ? &tseq : nullptr,
                      no_wrap ? &tpos : nullptr);
}

int nd_attn_decode_shared(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, uint32_t prefix_seq,
                          uint32_t prefix_rows, const void *q, const void *k, const void *v, const void *gate,
                          void *out) {
    int rc = check_call(h, layer, n, seq_ids, nullptr);
    if (rc) return rc;
    if (!q || !k || !v || !out) return fail(ND_ATTN_ERR_ARG, "null tensor");
    const nd_attn_config &c = h->cfg;
    if (prefix_seq >= c.max_seqs)
        return fail(ND_ATTN_ERR_RANGE, "prefix sequence %u >= max_seqs %u", prefix_seq, c.max_seqs);
    if (prefix_rows == 0 || prefix_rows > h->seqs[prefix_seq].pos)
        return fail(ND_ATTN_ERR_RANGE, "prefix rows %u: sequence %u holds %u written positions", prefix_rows,
                    prefix_seq, h->seqs[prefix_seq].pos);
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = seq_ids ? seq_ids[i] : i;
        const uint32_t pos = h->seqs[s].pos;
        if (pos >= c.window)
            return fail(ND_ATTN_ERR_RANGE, "sequence %u at position %u wraps the %u-slot ring", s, pos, c.window);
        if (pos < prefix_rows)
            return fail(ND_ATTN_ERR_RANGE, "sequence %u at position %u is inside the %u prefix rows", s, pos,
                        prefix_rows);
    }
    const int qk = (int)c.qk_head_dim, vd = (int)c.v_head_dim, nq = nda::nq_for_rep(h->rep);
    auto launch = [&](const AttnParams &P, uint32_t tpc, dim3 grid, int variant, float *part, size_t *smem) {
        switch (c.kv_dtype) {
        case ND_DT_I8:
            return nda::attend_shared_launch_i8(qk, vd, nq, P, prefix_seq, prefix_rows, tpc, grid, variant, part, smem,
                                                h->stream);
        case ND_DT_F32:
            return nda::attend_shared_launch_f32(qk, vd, nq, P, prefix_seq, prefix_rows, tpc, grid, variant, part, smem,
                                                 h->stream);
        case ND_DT_F16:
            return nda::attend_shared_launch_f16(qk, vd, nq, P, prefix_seq, prefix_rows, tpc, grid, variant, part, smem,
                                                 h->stream);
        default:
            return nda::attend_shared_launch_bf16(qk, vd, nq, P, prefix_seq, prefix_rows, tpc, grid, variant, part, smem,
                                                  h->stream);
        }
    };
    DeviceGuard dg(c.device);
    int smem_max = 0;
    ND_CUDA(cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, c.device));
    // Variant 2 (one lane per query row over the prefix) where it is built
    // (head dims up to 64) and its f32 staging fits; else variant 1; else the
    // regular path, which gives the same results. By default a call of fewer
    // than kSharedMinItems (token, KV head) pairs takes the regular path: a
    // warp of the staging kernel serves 32 query rows over the whole prefix,
    // so a small call leaves most SMs idle (config 5 at 1024 requests: 0.72
    // against 0.74 ms per step; at 4096: 1.49 against 2.50).
    constexpr uint64_t kSharedMinItems = 8192;
    if (h->shared_variant == 0 && (uint64_t)n * c.n_kv_heads < kSharedMinItems)
        return nd_attn_decode(h, layer, n, seq_ids, q, k, v, gate, out);
    int variant = 0;
    size_t smem = 0;
    if (h->shared_variant != 1 && launch(AttnParams{}, 0, dim3(1), 2, nullptr, &smem) == cudaSuccess &&
        smem <= (size_t)smem_max && (reinterpret_cast<uintptr_t>(q) & 15u) == 0)
        variant = 2;
    else if (launch(AttnParams{}, 0, dim3(1), 1, nullptr, &smem) == cudaSuccess && smem <= (size_t)smem_max)
        variant = 1;
    if (!variant) return nd_attn_decode(h, layer, n, seq_ids, q, k, v, gate, out);
    if (c.qkv_conv_taps) {
        std::vector<nda::SeqSpan> sp;
        if (seq_ids) {
            sp.resize(n);
            for (uint32_t i = 0; i < n; i++) sp[i] = nda::SeqSpan{seq_ids[i], i, 1u};
        }
        rc = run_taps(h, layer, n, seq_ids ? sp.data() : nullptr, n, &q, &k, &v);
        if (rc) return rc;
    }
    const TokMeta *d_tok = nullptr;
    if (seq_ids) {
        std::vector<TokMeta> tok(n);
        for (uint32_t i = 0; i < n; i++) tok[i] = TokMeta{seq_ids[i], 0u, i};
        rc = upload_tok(h, tok);
        if (rc) return rc;
        d_tok = h->d_tok;
    }
    if (variant == 2) {
        rc = grow(&h->shared_part, &h->shared_part_cap, (size_t)n * c.n_heads * (c.v_head_dim + 2));
        if (rc) return rc;
    }
    AttnParams P = base_params(h, layer);
    P.q = q; P.k = k; P.v = v; P.gate = gate; P.out = out;
    P.tok = d_tok;
    P.n_tok = n;
    P.fuse_append = 1;
    // Tokens per CTA of the staging launch: the call's (token, KV head) pairs
    // over two CTAs per SM, a whole number of the CTA's warps (variant 2:
    // nda::kSharedPrefixWarps; variant 1: 8) x tokens per warp step.
    const uint32_t per_sm = 2u;
    const uint32_t tw = variant == 2 ? 32u / (uint32_t)nq : (nq >= 4 ? 1u : 4u / (uint32_t)nq);
    const uint32_t step = (variant == 2 ? (uint32_t)nda::kSharedPrefixWarps : 8u) * tw;
    const uint64_t ctas = (uint64_t)per_sm * (uint64_t)h->sm_count;
    const uint64_t want = ((uint64_t)n * c.n_kv_heads + ctas - 1) / ctas;
    const uint32_t tpc = (uint32_t)std::max<uint64_t>(step, (want + step - 1) / step * step);
    const dim3 grid(c.n_kv_heads, (n + tpc - 1) / tpc, 1);
    note_writer(h, (int)layer);
    ND_CUDA(launch(P, tpc, grid, variant, h->shared_part, nullptr));
    if (variant == 2) h->launches++;
    h->launches++;
    return ND_ATTN_OK;
}

}  // extern "C"

namespace {

// Head norm + RoPE of query rows (zcrms_heads / apply_rope on m->q,
// nd_model.c:2419-2421, 326-397), one warp per (token, query head), in the
// reference's statement order (warp_norm_rope), from src to dst (the same
// buffer when no conv taps ran). Tokens map through P.spans / P.tok as in the
// append kernels.
template <int QK>
__global__ void __launch_bounds__(128) rope_q_kernel(const void *src, void *dst, const AttnParams P) {
    const int lane = (int)(threadIdx.x & 31u);
    const size_t item = (size_t)blockIdx.x * 4u + (threadIdx.x >> 5);
    if (item >= (size_t)P.n_tok * P.n_heads) return;
    const uint32_t tok = (uint32_t)(item / P.n_heads), hq = (uint32_t)(item % P.n_heads);
    const TokMeta tm = nda::token_meta(P, tok);
    const uint32_t pos = P.state[tm.seq].pos + tm.off;
    if (pos >= P.max_pos) {
        if (lane == 0) nda::set_err(P.err, 2);
        return;
    }
    const size_t base = ((size_t)tm.row * P.n_heads + hq) * QK;
    nda::RopePairs<QK> x;
    nda::warp_load_pairs<QK>(x, src, P.act_dt, base, lane);
    nda::warp_norm_rope<QK>(x, P.rope + (size_t)pos * (QK / 2), P.qnorm, lane);
#pragma unroll
    for (int c = 0; c < nda::RopePairs<QK>::PPL; c++) {
        const int i = lane + 32 * c;
        if (i < QK / 2) {
            nda::act_store(dst, P.act_dt, base + i, x.a[c]);
            nda::act_store(dst, P.act_dt, base + i + QK / 2, x.b[c]);
        }
    }
}

}  // namespace

extern "C" {

int nd_attn_rope_append(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const uint32_t *len,
                        void *q, const void *k, const void *v) {
    int rc = check_call(h, layer, n, seq_ids, len);
    if (rc) return rc;
    if (!k || !v) return fail(ND_ATTN_ERR_ARG, "null tensor");
    DeviceGuard dg(h->cfg.device);
    const nd_attn_config &c = h->cfg;
    const uint32_t W = c.window;
    std::vector<uint32_t> cu(n);
    std::vector<nda::SeqSpan> spans;
    size_t total = 0;
    uint32_t maxlen = 0;
    bool wraps = false;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = seq_ids ? seq_ids[i] : i, l = len ? len[i] : 1u;
        cu[i] = (uint32_t)total;
        total += l;
        maxlen = std::max(maxlen, l);
        // Two tokens of the call on one slot: the later must win, as in the
        // reference's token-at-a-time order.
        if ((uint64_t)h->seqs[s].pos + l > W && l > W - h->seqs[s].n_sink) wraps = true;
        if (l) spans.push_back(nda::SeqSpan{s, cu[i], l});
    }
    if (total == 0) return ND_ATTN_OK;
    if (total > 0x7fffffffu / std::max(c.n_heads, c.n_kv_heads)) return fail(ND_ATTN_ERR_RANGE, "too many tokens");
    const void *qs = q;
    if (c.qkv_conv_taps) {
        rc = run_taps(h, layer, (uint32_t)spans.size(), spans.data(), (uint32_t)total, &qs, &k, &v);
        if (rc) return rc;
    }
    rc = grow(&h->d_spans, &h->spans_cap, spans.size());
    if (rc) return rc;
    ND_CUDA(cudaMemcpyAsync(h->d_spans, spans.data(), spans.size() * sizeof(nda::SeqSpan), cudaMemcpyHostToDevice,
                            h->stream));
    AttnParams P = base_params(h, layer);
    P.k = k;
    P.v = v;
    note_writer(h, (int)layer);
    if (!wraps) {
        P.spans = h->d_spans;
        P.n_spans = (uint32_t)spans.size();
        P.n_tok = (uint32_t)total;
        ND_CUDA(append_launch(h, P));
        h->launches++;
    } else {
        // Token by token (offset t of every sequence that has it), in order.
        for (uint32_t t = 0; t < maxlen; t++) {
            std::vector<TokMeta> tok;
            for (uint32_t i = 0; i < n; i++)
                if (t < (len ? len[i] : 1u)) tok.push_back(TokMeta{seq_ids ? seq_ids[i] : i, t, cu[i] + t});
            rc = upload_tok(h, tok);
            if (rc) return rc;
            AttnParams Pt = P;
            Pt.tok = h->d_tok;
            Pt.n_tok = (uint32_t)tok.size();
            ND_CUDA(append_launch(h, Pt));
            h->launches++;
        }
    }
    if (q) {
        AttnParams Pq = base_params(h, layer);
        Pq.spans = h->d_spans;
        Pq.n_spans = (uint32_t)spans.size();
        Pq.n_tok = (uint32_t)total;
        const unsigned blocks = (unsigned)((total * c.n_heads + 3) / 4);
        switch (c.qk_head_dim) {
        case 48: rope_q_kernel<48><<<blocks, 128, 0, h->stream>>>(qs, q, Pq); break;
        case 64: rope_q_kernel<64><<<blocks, 128, 0, h->stream>>>(qs, q, Pq); break;
        default: rope_q_kernel<128><<<blocks, 128, 0, h->stream>>>(qs, q, Pq); break;
        }
        ND_CUDA(cudaGetLastError());
        h->launches++;
    }
    return ND_ATTN_OK;
}

int nd_attn_prefill(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const uint32_t *len,
                    const void *q, const void *k, const void *v, const void *gate, void *out) {
    if (!len) return fail(ND_ATTN_ERR_ARG, "null len");
    int rc = check_call(h, layer, n, seq_ids, len);
    if (rc) return rc;
    if (!q || !k || !v || !out) return fail(ND_ATTN_ERR_ARG, "null tensor");
    DeviceGuard dg(h->cfg.device);
    const uint32_t W = h->cfg.window;
    size_t total = 0;
    uint32_t maxlen = 0;
    bool wraps = false;
    std::vector<uint32_t> cu(n);
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = seq_ids ? seq_ids[i] : i;
        cu[i] = (uint32_t)total;
        total += len[i];
        maxlen = std::max(maxlen, len[i]);
        if ((uint64_t)h->seqs[s].pos + len[i] > W) wraps = true;
    }
    if (total == 0) return ND_ATTN_OK;
    if (total > 0x7fffffffu / h->cfg.n_kv_heads) return fail(ND_ATTN_ERR_RANGE, "too many tokens");
    if (h->cfg.qkv_conv_taps) {
        std::vector<nda::SeqSpan> sp;
        for (uint32_t i = 0; i < n; i++)
            if (len[i]) sp.push_back(nda::SeqSpan{seq_ids ? seq_ids[i] : i, cu[i], len[i]});
        rc = run_taps(h, layer, (uint32_t)sp.size(), sp.data(), (uint32_t)total, &q, &k, &v);
        if (rc) return rc;
    }
    if (!wraps) {
        // Every new position gets its own slot and nothing a token reads is
        // overwritten: append all tokens, then attend causally.
        std::vector<nda::SeqSpan> spans;
        spans.reserve(n);
        for (uint32_t i = 0; i < n; i++) {
            const uint32_t s = seq_ids ? seq_ids[i] : i;
            if (!len[i]) continue;
            spans.push_back(nda::SeqSpan{s, cu[i], len[i]});
        }
        rc = grow(&h->d_spans, &h->spans_cap, spans.size());
        if (rc) return rc;
        ND_CUDA(cudaMemcpyAsync(h->d_spans, spans.data(), spans.size() * sizeof(nda::SeqSpan),
                                cudaMemcpyHostToDevice, h->stream));
        AttnParams P = base_params(h, layer);
        P.k = k; P.v = v; P.spans = h->d_spans; P.n_spans = (uint32_t)spans.size(); P.n_tok = (uint32_t)total;
        note_writer(h, (int)layer);
        ND_CUDA(append_launch(h, P));
        h->launches++;
        if (tc_prefill_ok(h, q)) return run_prefill_tc(h, layer, n, seq_ids, len, cu, total, q, gate, out);
        std::vector<uint32_t> vis(total), tseq(total), tpos(total);
        for (uint32_t i = 0; i < n; i++) {
            const uint32_t s = seq_ids ? seq_ids[i] : i;
            for (uint32_t t = 0; t < len[i]; t++) {
                vis[cu[i] + t] = h->seqs[s].pos + t + 1;   // no wrap: [0, pos]
                tseq[cu[i] + t] = s;
                tpos[cu[i] + t] = h->seqs[s].pos + t;
            }
        }
        return run_attend(h, layer, (uint32_t)total, nullptr, h->d_spans, (uint32_t)spans.size(), vis, 0, q, k, v,
                          gate, out, &tseq, &tpos);
    }
    // The ring wraps inside this call: a later token's slot can hold a position
    // an earlier token still reads, so run the reference's token-at-a-time
    // order (append, then attend) step by step.
    for (uint32_t t = 0; t < maxlen; t++) {
        std::vector<TokMeta> tok;
        std::vector<uint32_t> vis;
        for (uint32_t i = 0; i < n; i++) {
            if (t >= len[i]) continue;
            const uint32_t s = seq_ids ? seq_ids[i] : i;
            tok.push_back(TokMeta{s, t, cu[i] + t});
            vis.push_back(visit_count(h->seqs[s].pos + t, h->seqs[s].n_sink, W));
        }
        rc = upload_tok(h, tok);
        if (rc) return rc;
        rc = run_attend(h, layer, (uint32_t)tok.size(), h->d_tok, nullptr, 0, vis, 1, q, k, v, gate, out, nullptr,
                        nullptr);
        if (rc) return rc;
    }
    return ND_ATTN_OK;
}

}  // extern "C"

namespace {

// Device address of a host range the device can read and write in place
// (pinned and mapped, as cudaHostAlloc and cudaHostRegister memory is under
// unified addressing), checked at both ends; nullptr for pageable (or
// managed) memory, which the caller stages. Device memory is no host buffer:
// *bad is set.
char *mapped_alias(const void *p, size_t bytes, bool *bad) {
    const char *end[2] = {static_cast<const char *>(p), static_cast<const char *>(p) + bytes - 1};
    char *dev[2];
    for (int i = 0; i < 2; i++) {
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, end[i]) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        if (a.type == cudaMemoryTypeDevice) {
            *bad = true;
            return nullptr;
        }
        if (a.type != cudaMemoryTypeHost || !a.devicePointer) return nullptr;
        dev[i] = static_cast<char *>(a.devicePointer);
    }
    return dev[1] - dev[0] == (ptrdiff_t)(bytes - 1) ? dev[0] : nullptr;
}

int grow_hstage(nd_attn *h, size_t need) {
    if (need <= h->hstage_cap) return ND_ATTN_OK;
    if (h->hstage) cudaFreeHost(h->hstage);
    h->hstage = h->hstage_dev = nullptr;
    h->hstage_cap = 0;
    const size_t n = std::max(need, (size_t)1 << 16);
    if (cudaHostAlloc(reinterpret_cast<void **>(&h->hstage), n, cudaHostAllocMapped | cudaHostAllocPortable) !=
            cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void **>(&h->hstage_dev), h->hstage, 0) != cudaSuccess) {
        if (h->hstage) cudaFreeHost(h->hstage);
        h->hstage = h->hstage_dev = nullptr;
        return fail(ND_ATTN_ERR_NOMEM, "pinned staging of %zu bytes failed", n);
    }
    h->hstage_cap = n;
    return ND_ATTN_OK;
}

// Host-buffer decode. The inputs reach the device through one ingest launch
// reading mapped host memory: the caller's pinned buffers in place, pageable
// ones after a host copy into the handle's pinned staging. The attend launch
// that follows may start under the ingest grid (it streams K/V meanwhile) and
// writes the output straight into mapped host memory, the caller's own when
// it is pinned. No copy-engine transfer is on the path.
int run_host_decode(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const void *q, const void *k,
                    const void *v, const void *gate, void *out) {
    const size_t b[5] = {act_bytes(h, n, 0), act_bytes(h, n, 1), act_bytes(h, n, 2), gate ? act_bytes(h, n, 3) : 0,
                         act_bytes(h, n, 4)};
    const void *src[5] = {q, k, v, gate, out};
    char *alias[5] = {};
    size_t soff[5] = {}, doff[4] = {}, stot = 0, dtot = 0;
    for (int i = 0; i < 5; i++) {
        if (!b[i]) continue;
        bool bad = false;
        alias[i] = mapped_alias(src[i], b[i], &bad);
        if (bad) return fail(ND_ATTN_ERR_ARG, "host-buffer call given device memory (argument %d)", i);
        soff[i] = stot;
        if (!alias[i]) stot += (b[i] + 255) / 256 * 256;
        if (i < 4) {
            doff[i] = dtot;
            dtot += (b[i] + 255) / 256 * 256;
        }
    }
    int rc = grow_hstage(h, stot);
    if (!rc) rc = grow(reinterpret_cast<char **>(&h->dio), &h->dio_cap, dtot);
    if (rc) return rc;
    char *d = static_cast<char *>(h->dio);
    IngestParams I;
    memset(&I, 0, sizeof(I));
    for (int i = 0; i < 4; i++) {
        if (!b[i]) continue;
        const char *from = alias[i];
        if (!from) {
            memcpy(h->hstage + soff[i], src[i], b[i]);
            from = h->hstage_dev + soff[i];
        }
        const uintptr_t al = reinterpret_cast<uintptr_t>(from) | b[i];   // dio offsets are 256-aligned
        const uint32_t shift = (al & 15) == 0 ? 4 : (al & 3) == 0 ? 2 : 0;
        I.seg[I.n] = IngestSeg{from, d + doff[i], b[i] >> shift, shift};
        I.first[I.n + 1] = I.first[I.n] + (b[i] >> shift);
        I.n++;
    }
    const uint64_t units = I.first[I.n];
    const uint32_t grid = (uint32_t)std::min<uint64_t>((units + 255) / 256, (uint64_t)h->sm_count * 8);
    ingest_kernel<<<grid, 256, 0, h->stream>>>(I);
    h->launches++;
    note_writer(h, kNoLayer);
    rc = cudaGetLastError() == cudaSuccess ? ND_ATTN_OK : fail(ND_ATTN_ERR_CUDA, "ingest launch failed");
    if (!rc)
        rc = nd_attn_decode(h, layer, n, seq_ids, d + doff[0], d + doff[1], d + doff[2], gate ? d + doff[3] : nullptr,
                            alias[4] ? alias[4] : h->hstage_dev + soff[4]);
    // The staging must not be rewritten while a launch of this call may read it.
    const int src_rc = nd_attn_sync(h);
    if (rc) return rc;
    if (src_rc) return src_rc;
    if (!alias[4]) memcpy(out, h->hstage + soff[4], b[4]);
    return ND_ATTN_OK;
}

// Host-buffer form: q/k/v/gate/out live in host memory.
int run_host(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const uint32_t *len,
             const void *q, const void *k, const void *v, const void *gate, void *out) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    int rc = check_call(h, layer, n, seq_ids, len);
    if (rc) return rc;
    if (!q || !k || !v || !out) return fail(ND_ATTN_ERR_ARG, "null tensor");
    DeviceGuard dg(h->cfg.device);
    if (!len) return run_host_decode(h, layer, n, seq_ids, q, k, v, gate, out);
    size_t tokens = 0;
    for (uint32_t i = 0; i < n; i++) tokens += len ? len[i] : 1;
    const size_t b[5] = {act_bytes(h, tokens, 0), act_bytes(h, tokens, 1), act_bytes(h, tokens, 2),
                         gate ? act_bytes(h, tokens, 3) : 0, act_bytes(h, tokens, 4)};
    size_t off[5], total = 0;
    for (int i = 0; i < 5; i++) {
        off[i] = total;
        total += (b[i] + 255) / 256 * 256;
    }
    rc = grow(reinterpret_cast<char **>(&h->dio), &h->dio_cap, total);
    if (rc) return rc;
    char *d = static_cast<char *>(h->dio);
    const void *src[4] = {q, k, v, gate};
    for (int i = 0; i < 4; i++) {
        if (!b[i]) continue;
        // Pinned sources copy asynchronously; pageable ones are staged by the
        // driver before the call returns.
        ND_CUDA(cudaMemcpyAsync(d + off[i], src[i], b[i], cudaMemcpyHostToDevice, h->stream));
    }
    rc = len ? nd_attn_prefill(h, layer, n, seq_ids, len, d + off[0], d + off[1], d + off[2],
                               gate ? d + off[3] : nullptr, d + off[4])
             : nd_attn_decode(h, layer, n, seq_ids, d + off[0], d + off[1], d + off[2],
                              gate ? d + off[3] : nullptr, d + off[4]);
    if (rc) return rc;
    ND_CUDA(cudaMemcpyAsync(out, d + off[4], b[4], cudaMemcpyDeviceToHost, h->stream));
    return nd_attn_sync(h);
}

}  // namespace

extern "C" {

int nd_attn_decode_host(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const void *q,
                        const void *k, const void *v, const void *gate, void *out) {
    return run_host(h, layer, n, seq_ids, nullptr, q, k, v, gate, out);
}

int nd_attn_prefill_host(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const uint32_t *len,
                         const void *q, const void *k, const void *v, const void *gate, void *out) {
    if (!len) return fail(ND_ATTN_ERR_ARG, "null len");
    return run_host(h, layer, n, seq_ids, len, q, k, v, gate, out);
}

}  // extern "C"

// ---- allocation-free decode ------------------------------------------------------
namespace {

// Fixed split-KV scratch of nd_attn_decode_noalloc, part of the library's
// device image: [tickets: MAX_ITEMS ints][partial (m,l)][partial o]. In host
// code `g_noalloc_scratch` names a host-side stand-in, never a device address:
// the address is looked up per device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[ND_ATTN_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_addr[kMaxDevices];

// Device address of the fixed scratch on `dev` (which must be current);
// looked up once per device.
int noalloc_scratch(int dev, char **addr) {
    if (dev < 0 || dev >= kMaxDevices) return fail(ND_ATTN_ERR_ARG, "device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(ND_ATTN_ERR_CUDA, "cudaGetSymbolAddress of the fixed scratch failed: %s",
                        cudaGetErrorString(e));
        g_noalloc_addr[dev] = p;
    }
    *addr = static_cast<char *>(g_noalloc_addr[dev]);
    return ND_ATTN_OK;
}

}  // namespace

extern "C" {

int nd_attn_decode_noalloc(nd_attn *h, uint32_t layer, uint32_t n, const void *q, const void *k, const void *v,
                           const void *gate, void *out) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    if (!q || !k || !v || !out) return fail(ND_ATTN_ERR_ARG, "null tensor");
    if (layer >= h->cfg.n_layers) return fail(ND_ATTN_ERR_RANGE, "layer %u >= n_layers %u", layer, h->cfg.n_layers);
    if (n == 0 || n > h->cfg.max_seqs) return fail(ND_ATTN_ERR_RANGE, "%u sequences (max %u)", n, h->cfg.max_seqs);
    const uint32_t n_kv = h->cfg.n_kv_heads, W = h->cfg.window;
    const size_t items = (size_t)n * n_kv;
    if (items > ND_ATTN_NOALLOC_MAX_ITEMS)
        return fail(ND_ATTN_ERR_RANGE, "%u sequences x %u KV heads exceeds the %u (sequence, KV head) pairs "
                    "the fixed scratch serves", n, n_kv, ND_ATTN_NOALLOC_MAX_ITEMS);
    uint32_t jmax = 1;
    size_t rows = 0;
    for (uint32_t i = 0; i < n; i++) {
        const HostSeq &s = h->seqs[i];
        if ((uint64_t)s.pos + 1 > h->cfg.max_pos)
            return fail(ND_ATTN_ERR_RANGE, "sequence %u at position %u >= max_pos %u", i, s.pos, h->cfg.max_pos);
        const uint32_t j = visit_count(s.pos, s.n_sink, W);
        jmax = std::max(jmax, j);
        rows += (size_t)j * n_kv;
    }
    DeviceGuard dg(h->cfg.device);
    char *base = nullptr;
    int rc = noalloc_scratch(h->cfg.device, &base);
    if (rc) return rc;
    if (h->cfg.qkv_conv_taps) {   // the tap buffer was sized for max_seqs tokens at open: no allocation
        rc = run_taps(h, layer, n, nullptr, n, &q, &k, &v);
        if (rc) return rc;
    }
    const size_t nq = (size_t)nda::nq_for_rep(h->rep);
    const size_t vd = h->cfg.v_head_dim;
    const size_t ticket_bytes = (size_t)ND_ATTN_NOALLOC_MAX_ITEMS * sizeof(int);
    const size_t slot_bytes = nq * (vd + 2) * sizeof(float);
    const size_t slots = (ND_ATTN_NOALLOC_SCRATCH_BYTES - ticket_bytes - 256) / slot_bytes;
    uint32_t chunk, nsplit;
    choose_split(h, items, jmax, rows, ND_ATTN_NOALLOC_MAX_ITEMS, slots, &chunk, &nsplit);
    AttnParams P = base_params(h, layer);
    P.q = q; P.k = k; P.v = v; P.gate = gate; P.out = out;
    P.tok = nullptr;
    P.n_tok = n;
    P.chunk = chunk;
    P.max_splits = nsplit;
    P.fuse_append = 1;
    P.counters = reinterpret_cast<int *>(base);
    P.part_ml = reinterpret_cast<float *>(base + ticket_bytes);
    const size_t ml_bytes = (slots * nq * 2 * sizeof(float) + 255) / 256 * 256;
    P.part_o = reinterpret_cast<float *>(base + ticket_bytes + ml_bytes);
    if (nsplit > 1) ND_CUDA(cudaMemsetAsync(P.counters, 0, items * sizeof(int), h->stream));
    note_writer(h, (int)layer);
    ND_CUDA(attend_launch(h, P, dim3((unsigned)items, nsplit, 1)));
    h->launches++;
    return ND_ATTN_OK;
}

// ---- prefix ------------------------------------------------------------------
nd_attn_prefix *nd_attn_prefix_save(nd_attn *h, uint32_t seq) {
    if (check_seq(h, seq)) return nullptr;
    const HostSeq &s = h->seqs[seq];
    if (!s.has_snap || s.pos != s.snap_pos) {
        fail(ND_ATTN_ERR_ARG, "prefix_save needs a snapshot at the current position");
        return nullptr;
    }
    DeviceGuard dg(h->cfg.device);
    const nd_attn_config &c = h->cfg;
    const uint32_t live = std::min(s.snap_pos + 1u, c.window);
    const size_t krow = h->k_dim * h->kes, vrow = h->v_dim * h->kes, srow = c.n_kv_heads * sizeof(float);
    const bool sc = c.kv_dtype == ND_DT_I8;
    // prefix_copy's order (nd_model.c:1493-1529): live K, V (and scale) rows,
    // then the snapshot's tap histories.
    const size_t hist_bytes = h->hist_seq * sizeof(float);
    const size_t bytes = (size_t)c.n_layers * live * (krow + vrow + (sc ? 2 * srow : 0)) + hist_bytes;
    nd_attn_prefix *p = new nd_attn_prefix();
    p->owner = h; p->pos = s.snap_pos; p->sink = s.n_sink; p->live = live; p->bytes = bytes;
    if (cudaMalloc(&p->dev, std::max<size_t>(bytes, 4)) != cudaSuccess) {
        fail(ND_ATTN_ERR_NOMEM, "prefix allocation of %zu bytes failed", bytes);
        delete p;
        return nullptr;
    }
    CacheView cv = layer_view(h, 0);
    char *dst = static_cast<char *>(p->dev);
    struct Part { void *base; size_t row; } parts[4] = {{h->kc, krow}, {h->vc, vrow}, {h->ks, srow}, {h->vs, srow}};
    for (int i = 0; i < (sc ? 4 : 2); i++) {
        note_writer(h, kAllLayers);
        rows_copy_kernel<<<dim3(std::min<uint32_t>(live, 1024u), c.n_layers), 128, 0, h->stream>>>(
            static_cast<char *>(parts[i].base), h->rows_per_layer * parts[i].row, dst, live * parts[i].row,
            (uint32_t)(parts[i].row / 4), live, cv, seq, 0, 0, nullptr);
        h->launches++;
        dst += (size_t)c.n_layers * live * parts[i].row;
    }
    if (hist_bytes)
        cudaMemcpyAsync(dst, h->d_snaphist + seq * h->hist_seq, hist_bytes, cudaMemcpyDeviceToDevice, h->stream);
    if (cudaStreamSynchronize(h->stream) != cudaSuccess) {
        fail(ND_ATTN_ERR_CUDA, "prefix copy failed: %s", cudaGetErrorString(cudaGetLastError()));
        cudaFree(p->dev);
        delete p;
        return nullptr;
    }
    return p;
}

int nd_attn_prefix_restore(nd_attn *h, uint32_t seq, const nd_attn_prefix *p) {
    if (!p || !h || p->owner != h) return fail(ND_ATTN_ERR_ARG, "prefix belongs to another handle");
    int rc = check_seq(h, seq);
    if (rc) return rc;
    DeviceGuard dg(h->cfg.device);
    const nd_attn_config &c = h->cfg;
    HostSeq &s = h->seqs[seq];
    s.snap_pos = p->pos;
    s.n_sink = p->sink;
    const size_t krow = h->k_dim * h->kes, vrow = h->v_dim * h->kes, srow = c.n_kv_heads * sizeof(float);
    const bool sc = c.kv_dtype == ND_DT_I8;
    CacheView cv = layer_view(h, 0);
    char *src = static_cast<char *>(p->dev);
    struct Part { void *base; size_t row; } parts[4] = {{h->kc, krow}, {h->vc, vrow}, {h->ks, srow}, {h->vs, srow}};
    for (int i = 0; i < (sc ? 4 : 2); i++) {
        note_writer(h, kAllLayers);
        rows_copy_kernel<<<dim3(std::min<uint32_t>(p->live, 1024u), c.n_layers), 128, 0, h->stream>>>(
            static_cast<char *>(parts[i].base), h->rows_per_layer * parts[i].row, src, p->live * parts[i].row,
            (uint32_t)(parts[i].row / 4), p->live, cv, seq, 0, 1,
            i <= 1 && c.kv_dtype == ND_DT_BF16 ? h->d_vbig : nullptr);
        h->launches++;
        src += (size_t)c.n_layers * p->live * parts[i].row;
    }
    if (h->hist_seq)
        ND_CUDA(cudaMemcpyAsync(h->d_snaphist + seq * h->hist_seq, src, h->hist_seq * sizeof(float),
                                cudaMemcpyDeviceToDevice, h->stream));
    ND_CUDA(cudaGetLastError());
    s.has_snap = 1;
    s.pos = s.snap_pos;  // nd_model_rewind
    rc = hist_copy(h, seq, false);
    return rc ? rc : push_state(h, seq);
}

void nd_attn_prefix_free(nd_attn_prefix *p) {
    if (!p) return;
    if (p->owner) {
        DeviceGuard dg(p->owner->cfg.device);
        cudaFree(p->dev);
    }
    delete p;
}

int nd_attn_prefix_read(const nd_attn_prefix *p, void *host, size_t cap, size_t *bytes, uint32_t *pos,
                        uint32_t *n_sink) {
    if (!p) return fail(ND_ATTN_ERR_ARG, "null prefix");
    if (bytes) *bytes = p->bytes;
    if (pos) *pos = p->pos;
    if (n_sink) *n_sink = p->sink;
    if (host && cap >= p->bytes && p->bytes) {
        DeviceGuard dg(p->owner->cfg.device);
        ND_CUDA(cudaStreamSynchronize(p->owner->stream));
        ND_CUDA(cudaMemcpy(host, p->dev, p->bytes, cudaMemcpyDeviceToHost));
    }
    return ND_ATTN_OK;
}

// ---- cache access ----------------------------------------------------------------
static int cache_io(nd_attn *h, uint32_t layer, uint32_t seq, uint32_t slot0, uint32_t n_slots, void *k, void *v,
                    float *k_scale, float *v_scale, int to_cache) {
    int rc = check_seq(h, seq);
    if (rc) return rc;
    if (layer >= h->cfg.n_layers) return fail(ND_ATTN_ERR_RANGE, "layer %u", layer);
    if ((uint64_t)slot0 + n_slots > h->cfg.window) return fail(ND_ATTN_ERR_RANGE, "slots beyond the window");
    if (n_slots == 0) return ND_ATTN_OK;
    DeviceGuard dg(h->cfg.device);
    const nd_attn_config &c = h->cfg;
    const size_t krow = h->k_dim * h->kes, vrow = h->v_dim * h->kes, srow = c.n_kv_heads * sizeof(float);
    const bool sc = c.kv_dtype == ND_DT_I8;
    const size_t need = (size_t)n_slots * (krow + vrow + 2 * srow);
    rc = grow(reinterpret_cast<char **>(&h->dio), &h->dio_cap, need + 1024);
    if (rc) return rc;
    char *d = static_cast<char *>(h->dio);
    CacheView cv = layer_view(h, layer);
    struct Part { void *cache; void *user; size_t row; } parts[4] = {
        {cv.k, k, krow}, {cv.v, v, vrow}, {cv.ks, k_scale, srow}, {cv.vs, v_scale, srow}};
    size_t off = 0;
    for (int i = 0; i < 4; i++) {
        if (i >= 2 && !sc) break;
        if (!parts[i].user) continue;
        const size_t nb = n_slots * parts[i].row;
        char *dense = to_cache ? static_cast<char *>(parts[i].user) : d + off;
        note_writer(h, kAllLayers);
        rows_copy_kernel<<<dim3(std::min<uint32_t>(n_slots, 4096u), 1), 128, 0, h->stream>>>(
            static_cast<char *>(parts[i].cache), 0, dense, 0, (uint32_t)(parts[i].row / 4), n_slots, cv, seq,
            slot0, to_cache, to_cache && i <= 1 ? cv.vbig : nullptr);
        h->launches++;
        ND_CUDA(cudaGetLastError());
        if (!to_cache) ND_CUDA(cudaMemcpyAsync(parts[i].user, d + off, nb, cudaMemcpyDeviceToHost, h->stream));
        off += (nb + 255) / 256 * 256;
    }
    return nd_attn_sync(h);
}

int nd_attn_read_cache(nd_attn *h, uint32_t layer, uint32_t seq, uint32_t slot0, uint32_t n_slots, void *k,
                       void *v, float *k_scale, float *v_scale) {
    return cache_io(h, layer, seq, slot0, n_slots, k, v, k_scale, v_scale, 0);
}

int nd_attn_write_cache(nd_attn *h, uint32_t layer, uint32_t seq, uint32_t slot0, uint32_t n_slots,
                        const void *k, const void *v, const float *k_scale, const float *v_scale) {
    return cache_io(h, layer, seq, slot0, n_slots, const_cast<void *>(k), const_cast<void *>(v),
                    const_cast<float *>(k_scale), const_cast<float *>(v_scale), 1);
}

int nd_attn_set_block_table(nd_attn *h, uint32_t seq, const int32_t *pages) {
    int rc = check_seq(h, seq);
    if (rc) return rc;
    if (!h->cfg.block_size) return fail(ND_ATTN_ERR_ARG, "handle is not paged");
    if (!pages) return fail(ND_ATTN_ERR_ARG, "null page list");
    for (uint32_t i = 0; i < h->blocks_per_seq; i++)
        if (pages[i] < 0 || (uint32_t)pages[i] >= h->cfg.n_blocks)
            return fail(ND_ATTN_ERR_RANGE, "page %d out of range", pages[i]);
    DeviceGuard dg(h->cfg.device);
    ND_CUDA(cudaMemcpyAsync(h->d_btab + (size_t)seq * h->blocks_per_seq, pages, h->blocks_per_seq * sizeof(int32_t),
                            cudaMemcpyHostToDevice, h->stream));
    return nd_attn_sync(h);
}

int nd_attn_sync(nd_attn *h) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    DeviceGuard dg(h->cfg.device);
    // Kernels store their status straight into mapped host memory: after the
    // stream has drained it is readable with no copy.
    ND_CUDA(cudaStreamSynchronize(h->stream));
    const int err = *reinterpret_cast<volatile int *>(h->err_host);
    if (err) {
        *reinterpret_cast<volatile int *>(h->err_host) = 0;
        cudaMemset(h->counters, 0, h->counter_cap * sizeof(int));
        return fail(err == 3 ? ND_ATTN_ERR_TIMEOUT : ND_ATTN_ERR_RANGE,
                    "device reported status %d (position/state out of range or bounded wait expired)", err);
    }
    return ND_ATTN_OK;
}

int nd_attn_selftest_wait(nd_attn *h, uint32_t limit_us) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    if (limit_us == 0 || limit_us > 1000000u) return fail(ND_ATTN_ERR_RANGE, "limit_us %u outside [1, 1000000]", limit_us);
    DeviceGuard dg(h->cfg.device);
    // 2000 cycles per microsecond bounds the wait from above at SM clocks up
    // to 2 GHz (B200: 1965 MHz at most).
    wait_expiry_kernel<<<1, 32, 0, h->stream>>>(h->d_err, (long long)limit_us * 2000);
    h->launches++;
    ND_CUDA(cudaGetLastError());
    return nd_attn_sync(h);
}

void *nd_attn_stream(nd_attn *h) { return h ? static_cast<void *>(h->stream) : nullptr; }

int nd_attn_set_stream(nd_attn *h, void *stream) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    DeviceGuard dg(h->cfg.device);
    ND_CUDA(cudaStreamSynchronize(h->stream));
    h->stream = stream ? static_cast<cudaStream_t>(stream) : h->own;
    return ND_ATTN_OK;
}

uint64_t nd_attn_launch_count(const nd_attn *h) { return h ? h->launches : 0; }

const char *nd_attn_last_error(void) { return g_err.c_str(); }

const char *nd_attn_version(void) {
    static char buf[64];
    if (!buf[0]) snprintf(buf, sizeof(buf), "nd_attn 0.1 sm_100a cudart %d", CUDART_VERSION);
    return buf;
}

}  // extern "C"

// ============================================================ head-sharded decode
namespace {

constexpr uint32_t kGatherMagic = 0x4147444eu;   // "NDGA"
constexpr uint32_t kGatherVersion = 2;

// The record one rank hands to every other rank (ND_ATTN_GATHER_BLOB_BYTES).
struct GatherBlob {
    uint32_t magic, version, rank, world;
    uint32_t max_tokens, row_words;   // gathered row: 8-byte words of {4 data bytes, epoch}
    uint64_t slot_bytes;
    uint32_t out_dtype, pad0;
    uint8_t uuid[16];   // the rank's GPU (cudaDeviceProp::uuid)
    uint8_t ipc[64];    // cudaIpcMemHandle_t of the rank's gather buffer
    uint8_t pad1[8];
};
static_assert(sizeof(GatherBlob) == ND_ATTN_GATHER_BLOB_BYTES, "gather blob layout");
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");

// Ends a gathered call on this rank: copies the data half of every word of
// this rank's slot to `out` once the word carries the call's epoch (each
// word is one 64-bit store of some rank's attend kernel, so a word with the
// epoch is complete), polling with a bounded wait (~2 s; on expiry status 3,
// ND_ATTN_ERR_TIMEOUT). Launched as a programmatic dependent of the attend
// launch, it lets the next launch start at once and copies rows as they
// arrive, while the attend launch still runs; it waits for that launch to
// complete only at its end, so its own completion implies that launch's.
// n_words is even and `out` 8-byte aligned.
__global__ void gather_wait_kernel(const unsigned long long *slot, uint2 *out, size_t n_words, uint32_t epoch,
                                   int *err) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const long long t0 = clock64();
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words / 2; i += stride) {
        unsigned long long a, b;
        for (;;) {
            asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(slot + 2 * i) : "memory");
            if ((uint32_t)(a >> 32) == epoch && (uint32_t)(b >> 32) == epoch) break;
            if (clock64() - t0 > nda::kTimeoutCycles) {
                nda::set_err(err, 3);
                i = n_words;   // stop this thread
                break;
            }
            __nanosleep(64);
        }
        if (i < n_words / 2) out[i] = make_uint2((uint32_t)a, (uint32_t)b);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

int gather_check(const GatherBlob *b, uint32_t world, uint32_t rank) {
    if (world < 1 || world > (uint32_t)nda::kMaxGather)
        return fail(ND_ATTN_ERR_ARG, "world %u outside [1, %d]", world, nda::kMaxGather);
    if (rank >= world) return fail(ND_ATTN_ERR_ARG, "rank %u >= world %u", rank, world);
    static const uint8_t zero[16] = {0};
    for (uint32_t i = 0; i < world; i++) {
        if (b[i].magic != kGatherMagic || b[i].version != kGatherVersion)
            return fail(ND_ATTN_ERR_ARG, "record %u is not a gather record of this library version", i);
        if (b[i].rank != i || b[i].world != world)
            return fail(ND_ATTN_ERR_ARG, "record %u comes from rank %u of %u (records must be in rank order)", i,
                        b[i].rank, b[i].world);
        if (b[i].max_tokens != b[0].max_tokens || b[i].row_words != b[0].row_words ||
            b[i].slot_bytes != b[0].slot_bytes || b[i].out_dtype != b[0].out_dtype)
            return fail(ND_ATTN_ERR_ARG, "rank %u's handle has another geometry than rank 0's", i);
        for (uint32_t j = 0; j < i; j++)
            if (memcmp(b[i].uuid, zero, 16) && !memcmp(b[i].uuid, b[j].uuid, 16))
                return fail(ND_ATTN_ERR_ARG, "ranks %u and %u share one GPU (one rank per GPU is required: the "
                            "ranks' kernels wait for one another)", j, i);
    }
    return ND_ATTN_OK;
}

}  // namespace

extern "C" {

int nd_attn_gather_check(const void *blobs, uint32_t world, uint32_t rank) {
    if (!blobs) return fail(ND_ATTN_ERR_ARG, "null records");
    return gather_check(static_cast<const GatherBlob *>(blobs), world, rank);
}

int nd_attn_gather_init(nd_attn *h, uint32_t rank, uint32_t world, void *blob) {
    if (!h || !blob) return fail(ND_ATTN_ERR_ARG, "null argument");
    if (h->g_world) return fail(ND_ATTN_ERR_ARG, "the handle is already set up for a gather");
    if (world < 1 || world > (uint32_t)nda::kMaxGather || rank >= world)
        return fail(ND_ATTN_ERR_ARG, "rank %u of world %u (world at most %d)", rank, world, nda::kMaxGather);
    const nd_attn_config &c = h->cfg;
    DeviceGuard dg(c.device);
    // A word carries one f32 or two 16-bit output elements.
    const size_t elems = (size_t)world * c.n_heads * c.v_head_dim;
    const size_t words = c.out_dtype == ND_DT_F32 ? elems : elems / 2;
    const size_t slot_bytes = ((size_t)c.max_seqs * words * 8 + 255) / 256 * 256;
    if (words > 0x7fffffffu) return fail(ND_ATTN_ERR_RANGE, "gathered row too large");
    if (cudaMalloc(&h->g_buf, 2 * slot_bytes) != cudaSuccess) {
        cudaGetLastError();
        h->g_buf = nullptr;
        return fail(ND_ATTN_ERR_NOMEM, "gather buffer of %zu bytes", 2 * slot_bytes);
    }
    ND_CUDA(cudaMemset(h->g_buf, 0, 2 * slot_bytes));   // epoch 0 is never used
    GatherBlob b;
    memset(&b, 0, sizeof(b));
    b.magic = kGatherMagic;
    b.version = kGatherVersion;
    b.rank = rank;
    b.world = world;
    b.max_tokens = c.max_seqs;
    b.row_words = (uint32_t)words;
    b.slot_bytes = slot_bytes;
    b.out_dtype = (uint32_t)c.out_dtype;
    cudaDeviceProp prop;
    ND_CUDA(cudaGetDeviceProperties(&prop, c.device));
    memcpy(b.uuid, &prop.uuid, 16);
    cudaIpcMemHandle_t ipc;
    ND_CUDA(cudaIpcGetMemHandle(&ipc, h->g_buf));
    memcpy(b.ipc, &ipc, 64);
    memcpy(blob, &b, sizeof(b));
    h->g_world = world;
    h->g_rank = rank;
    h->g_words = (uint32_t)words;
    h->g_slot_bytes = slot_bytes;
    return ND_ATTN_OK;
}

int nd_attn_gather_attach(nd_attn *h, const void *blobs) {
    if (!h || !blobs) return fail(ND_ATTN_ERR_ARG, "null argument");
    if (!h->g_world) return fail(ND_ATTN_ERR_ARG, "nd_attn_gather_init has not run on this handle");
    if (h->g_ready) return fail(ND_ATTN_ERR_ARG, "the handle is already attached");
    const GatherBlob *b = static_cast<const GatherBlob *>(blobs);
    int rc = gather_check(b, h->g_world, h->g_rank);
    if (rc) return rc;
    if (b[0].row_words != h->g_words || b[0].slot_bytes != h->g_slot_bytes ||
        b[0].out_dtype != (uint32_t)h->cfg.out_dtype)
        return fail(ND_ATTN_ERR_ARG, "the records' geometry differs from this handle's");
    DeviceGuard dg(h->cfg.device);
    for (uint32_t p = 0; p < h->g_world; p++) {
        if (p == h->g_rank) {
            h->g_peer[p] = h->g_buf;
            continue;
        }
        cudaIpcMemHandle_t ipc;
        memcpy(&ipc, b[p].ipc, 64);
        void *ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, ipc, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (uint32_t q = 0; q < p; q++)
                if (q != h->g_rank && h->g_peer[q]) cudaIpcCloseMemHandle(h->g_peer[q]);
            memset(h->g_peer, 0, sizeof(h->g_peer));
            return fail(ND_ATTN_ERR_CUDA, "cudaIpcOpenMemHandle of rank %u's buffer: %s", p, cudaGetErrorString(e));
        }
        h->g_peer[p] = static_cast<char *>(ptr);
    }
    h->g_ready = true;
    return ND_ATTN_OK;
}

int nd_attn_decode_gather(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const void *q,
                          const void *k, const void *v, const void *gate, void *out) {
    if (!h) return fail(ND_ATTN_ERR_ARG, "null handle");
    if (!h->g_ready) return fail(ND_ATTN_ERR_ARG, "nd_attn_gather_attach has not run on this handle");
    if (!out) return fail(ND_ATTN_ERR_ARG, "null tensor");
    if (reinterpret_cast<uintptr_t>(out) & 7u) return fail(ND_ATTN_ERR_ARG, "out must be 8-byte aligned");
    if (n > h->cfg.max_seqs) return fail(ND_ATTN_ERR_RANGE, "%u sequences (max %u)", n, h->cfg.max_seqs);
    DeviceGuard dg(h->cfg.device);
    // Every rank numbers its gathered calls alike: 1, 2, ... (0 skipped at the
    // wrap; the slots alternate by the number's parity).
    const uint32_t prev = h->g_epoch;
    h->g_epoch = prev + 1 ? prev + 1 : 1;
    const uint32_t epoch = h->g_epoch, slot = epoch & 1u;
    nda::GatherView g{};
    g.G = h->g_world;
    g.col0 = h->g_rank * h->cfg.n_heads * h->cfg.v_head_dim;
    g.row_elems = h->g_world * h->cfg.n_heads * h->cfg.v_head_dim;
    g.epoch = epoch;
    for (uint32_t p = 0; p < h->g_world; p++)
        g.slot[p] = reinterpret_cast<unsigned long long *>(h->g_peer[p] + slot * h->g_slot_bytes);
    h->gth_call = g;
    int rc = nd_attn_decode(h, layer, n, seq_ids, q, k, v, gate, out);
    h->gth_call = nda::GatherView{};
    if (rc) {
        h->g_epoch = prev;   // refused before its attend launch: the ranks' call numbers stay equal
        return rc;
    }
    // The wait-and-copy kernel, a programmatic dependent of the attend launch
    // (which may still be writing this layer's cache, so the writer record is
    // left as it is).
    const size_t n_words = (size_t)n * h->g_words;
    const unsigned threads = 256;
    const unsigned blocks = (unsigned)std::max<size_t>(
        1, std::min<size_t>((n_words / 2 + threads - 1) / threads, (size_t)h->sm_count));
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(blocks);
    lc.blockDim = dim3(threads);
    lc.stream = h->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    const unsigned long long *own = reinterpret_cast<const unsigned long long *>(h->g_buf + slot * h->g_slot_bytes);
    ND_CUDA(cudaLaunchKernelEx(&lc, gather_wait_kernel, own, static_cast<uint2 *>(out), n_words, epoch, h->d_err));
    h->launches++;
    return ND_ATTN_OK;
}

}  // extern "C"

const nd_attn_ops *nd_attn_cuda_ops(void) {
    static const nd_attn_ops ops = {
        ND_ATTN_OPS_VERSION,   nd_attn_open,          nd_attn_close,        nd_attn_set_head_norm,
        nd_attn_reset,         nd_attn_set_sink,      nd_attn_snapshot,     nd_attn_rewind,
        nd_attn_advance,       nd_attn_decode,        nd_attn_prefill,      nd_attn_decode_host,
        nd_attn_prefill_host,  nd_attn_prefix_save,   nd_attn_prefix_restore, nd_attn_prefix_free,
        nd_attn_sync,          nd_attn_last_error,    nd_attn_set_conv_taps,
    };
    return &ops;
}

// Error reporting for the library's other translation units (nd_cq.cu): the
// same per-thread message nd_attn_last_error() returns.
namespace nda {
int report_error(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}
}  // namespace nda
