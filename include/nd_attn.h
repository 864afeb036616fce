/* nd_attn.h - B200 (sm_100a) attention hot path of the Needle engine, as a C ABI.
 *
 * This library replaces the attention section of the reference engine's
 * forward pass: per-head ZC-RMSNorm + NeoX RoPE, the KV-cache append into the
 * sink-plus-ring slot layout, and the online-softmax attention over the cache,
 * plus the schema-prefix machinery (sink pinning, snapshot/rewind, prefix
 * save/restore). Reference seam: the static `attention()` of
 * engine/src/nd_model.c:2382, lines 2419-2483 (norm+RoPE 2419-2422, KV store
 * 2426-2449, attn_heads dispatch 2451-2483).
 *
 * Conventions (copied from the reference engine so callers need no new rules):
 *  - 0 on success, a negative code on failure (nd_model_open returns -10..-13,
 *    engine/src/nd_model.c:760-761,766-768,1205-1221); -1 for an argument or an
 *    owner mismatch (nd_model_prefix_restore, nd_model.c:1545); NULL for a failed
 *    prefix allocation (nd_model_prefix_save, nd_model.c:1531-1535).
 *  - The handle owns every device buffer (caches, scales, state, scratch), as
 *    nd_model owns its caches (nd_model.c:1195-1198, freed 1262-1300). Tensor
 *    arguments are caller-owned.
 *  - One caller thread per handle, like the reference step API. Every call is
 *    stream-ordered on the handle's CUDA stream; the plain entry points return
 *    after enqueueing, `*_host` entry points and state/prefix calls return after
 *    the stream has drained. nd_attn_sync() waits explicitly.
 *  - Decode and non-wrapping prefill kernels of 16-bit caches are launched with
 *    programmatic stream serialization: one may begin under the tail of the
 *    previous kernel on the stream and stream its own layer's K/V early, but it
 *    reads the caller's tensors and writes `out` only after that kernel has
 *    completed, so stream order holds for everything the caller can see.
 *  - No torch or C++ types cross this boundary: plain pointers and sizes.
 *
 * Tensor layouts (row-major, elements of `act_dtype` unless stated):
 *  q    [tokens][n_heads][qk_head_dim]
 *  k    [tokens][n_kv_heads][qk_head_dim]
 *  v    [tokens][n_kv_heads][v_head_dim]
 *  gate [tokens][n_heads][v_head_dim]      pre-sigmoid, nullable (= gate of 1)
 *  out  [tokens][n_heads][v_head_dim]      elements of `out_dtype`
 * Tokens of one call are packed sequence after sequence (`len[i]` tokens for
 * the i-th listed sequence; decode = one token each).
 *
 * KV cache, per layer: rows of [n_kv_heads][head_dim] elements of `kv_dtype`,
 * one row per slot, exactly the reference layout k_cache[layer][window][k_dim]
 * (engine/include/nd_model.h:132-137) for each sequence; with int8 KV a float
 * scale per (slot, KV head) as k_scale[layer][window][n_kv_heads]. A position
 * p lives in slot kv_slot(p) = p < n_sink ? p : n_sink + (p-n_sink) % (window-n_sink)
 * (nd_model.c:1304-1309). Paged mode (block_size > 0) splits each sequence's
 * window into block_size-slot pages placed through a per-sequence block table.
 */
#ifndef ND_ATTN_H
#define ND_ATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ND_ATTN_API __attribute__((visibility("default")))
#else
#define ND_ATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ---------------------------------------------------- */
#define ND_ATTN_OK            0
#define ND_ATTN_ERR_ARG      (-1)   /* bad argument, owner mismatch (nd_model.c:1545) */
#define ND_ATTN_ERR_GEOM     (-10)  /* geometry outside the supported caps (nd_model.c:760) */
#define ND_ATTN_ERR_NOMEM    (-12)  /* device/host allocation failed (nd_model.c:1219) */
#define ND_ATTN_ERR_CUDA     (-14)  /* CUDA runtime error; see nd_attn_last_error() */
#define ND_ATTN_ERR_RANGE    (-15)  /* sequence id, slot count or position out of range */
#define ND_ATTN_ERR_TIMEOUT  (-16)  /* a bounded device-side wait expired */
#define ND_ATTN_ERR_NOGPU    (-17)  /* no usable sm_100 device */

/* ---- element types ---------------------------------------------------- */
typedef enum {
    ND_DT_I8   = 0,   /* KV only: symmetric int8 + fp32 scale per (slot, KV head) */
    ND_DT_F32  = 1,
    ND_DT_F16  = 2,
    ND_DT_BF16 = 3
} nd_attn_dtype;

/* ---- configuration ------------------------------------------------------
 * Geometry fields carry the reference's names (nd_model.h:98-99).
 * Supported head dims: (qk_head_dim, v_head_dim) in {(48,64), (64,64),
 * (128,128)}; n_heads % n_kv_heads == 0 with n_heads/n_kv_heads <= 8
 * (ND_KV_REP_CAP, nd_model.h:245). */
typedef struct {
    uint32_t n_layers;
    uint32_t n_heads;        /* query heads */
    uint32_t n_kv_heads;
    uint32_t qk_head_dim;
    uint32_t v_head_dim;
    uint32_t window;         /* KV slots per sequence, sinks + ring (nd_model.c:757) */
    uint32_t max_seqs;       /* independent sequences held by the handle */
    uint32_t block_size;     /* 0: contiguous window per sequence; else slots per page */
    uint32_t n_blocks;       /* pages per layer in paged mode (0: max_seqs*window/block_size) */
    uint32_t max_pos;        /* RoPE table length: positions must stay below it (0: window) */
    float    rope_theta;     /* nd_cact_header.rope_theta (nd_cact.h:66) */
    int32_t  kv_dtype;       /* nd_attn_dtype */
    int32_t  act_dtype;      /* q/k/v/gate element type: F32, F16 or BF16 */
    int32_t  out_dtype;      /* out element type: F32, F16 or BF16 */
    int32_t  device;         /* CUDA device ordinal */
    uint32_t qkv_conv_taps;  /* 0, or the short causal convolution over q/k/v
                              * projections (nd_cact_header.qkv_conv_taps,
                              * nd_cact.h:55), at most 4 taps */
} nd_attn_config;

typedef struct nd_attn nd_attn;
typedef struct nd_attn_prefix nd_attn_prefix;

/* Fills `cfg` with the defaults of a single-sequence fp32 handle. */
ND_ATTN_API void nd_attn_config_init(nd_attn_config *cfg);

/* Replaces nd_model_open's cache allocation (nd_model.c:1138-1198) and the
 * rope_inv table (nd_model.c:1233-1236): allocates caches, scales, per-sequence
 * state and scratch on `cfg->device`, uploads the RoPE cos/sin table for
 * positions [0, max_pos). Every sequence starts reset (nd_model_reset). */
ND_ATTN_API int  nd_attn_open(const nd_attn_config *cfg, nd_attn **out);
/* Replaces nd_model_close's cache release (nd_model.c:1262-1300). */
ND_ATTN_API void nd_attn_close(nd_attn *h);

/* Per-layer ZC-RMSNorm scales applied before RoPE, the layer's q_norm and
 * k_norm tensors (nd_model.c:2419-2422, zcrms_head_rows 326-365), each
 * qk_head_dim floats (host). NULL for both = pure RoPE for that layer
 * (apply_rope, nd_model.c:381-397). */
ND_ATTN_API int  nd_attn_set_head_norm(nd_attn *h, uint32_t layer,
                           const float *q_scale, const float *k_scale);

/* Per-layer tap weights of the QKV short causal convolution, the layer's
 * archive tensors 4, 5 and 6 staged as floats (nd_model.c:782-823):
 * wq [taps][n_heads * qk_head_dim], wk [taps][n_kv_heads * qk_head_dim],
 * wv [taps][n_kv_heads * v_head_dim], element (j, i) at j * dim + i (host).
 * With taps configured, the q/k/v every decode and prefill call takes are the
 * raw projections: each token's column i becomes
 *   0 + w[0][i]*x(pos)[i] + w[1][i]*x(pos-1)[i] + ...  over min(taps, pos+1)
 * taps, separately rounded in ascending tap order (tap_projection /
 * tap_rows, nd_model.c:2361-2379, 1753-1802), before the head norm and RoPE.
 * The per-sequence history of raw projections is kept on the device; reset
 * clears it, snapshot / rewind / prefix_save / prefix_restore carry it like
 * nd_model_snapshot (nd_model.c:1395-1456). Layers start with w[0] = 1 and
 * the other taps 0. 16-bit activations: the convolved rows are rounded to
 * act_dtype. */
ND_ATTN_API int  nd_attn_set_conv_taps(nd_attn *h, uint32_t layer, const float *wq, const float *wk,
                           const float *wv);

/* ---- session state (per sequence) --------------------------------------- */
/* nd_model_reset (nd_model.c:1557-1581): pos = 0, n_sink = 0, no snapshot. */
ND_ATTN_API int  nd_attn_reset(nd_attn *h, uint32_t seq);
/* nd_model_set_sink (nd_model.c:1314-1321): n_sink = min(n, window - 64). */
ND_ATTN_API int  nd_attn_set_sink(nd_attn *h, uint32_t seq, uint32_t n);
/* nd_model_snapshot (nd_model.c:1395-1434): pins [0, pos) as sinks and
 * remembers pos. */
ND_ATTN_API int  nd_attn_snapshot(nd_attn *h, uint32_t seq);
/* nd_model_rewind (nd_model.c:1436-1460): back to the snapshot position, or a
 * reset when there is none. */
ND_ATTN_API int  nd_attn_rewind(nd_attn *h, uint32_t seq);
/* Moves the position of `n` sequences on by len[i] tokens (NULL len = 1 each),
 * the `m->pos++` at the end of nd_model_step_hidden. seq_ids NULL = 0..n-1. */
ND_ATTN_API int  nd_attn_advance(nd_attn *h, uint32_t n, const uint32_t *seq_ids, const uint32_t *len);
ND_ATTN_API int  nd_attn_get_state(nd_attn *h, uint32_t seq, uint32_t *pos, uint32_t *n_sink);
/* Test/bench set-up of a synthetic session: sets pos and n_sink directly. */
ND_ATTN_API int  nd_attn_set_state(nd_attn *h, uint32_t seq, uint32_t pos, uint32_t n_sink);

/* ---- the hot path -------------------------------------------------------- */
/* Decode: one new token for each of `n` sequences at their current position.
 * Per sequence and layer: norm+RoPE of q and k, KV append at kv_slot(pos),
 * attention over sinks [0, min(n_sink,pos+1)) then the recent run ending at pos
 * (nd_model.c:2451-2481), sigmoid gate on the emit (attn_gate_emit,
 * nd_model.c:2091-2103). q/k/v/gate/out are DEVICE pointers. Does not advance. */
ND_ATTN_API int  nd_attn_decode(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids,
                    const void *q, const void *k, const void *v, const void *gate,
                    void *out);
/* Decode of `n` sequences that all begin with the same cache rows: the
 * requests of shared-prefix serving, each restored from one saved schema
 * prefix (nd_model_prefix_restore, nd_model.c:1543-1553, per request as in
 * esp32/main/main.c:281-315). Same arguments, work and results as
 * nd_attn_decode, given that cache rows [0, prefix_rows) of every listed
 * sequence hold the same K/V as those of sequence `prefix_seq` (block tables
 * that map the same pages, or prefix_restore of the same image). The library
 * reads those rows once per CTA from prefix_seq (staged in shared memory and
 * scored against many requests' queries) instead of once per request; each
 * request's own rows [prefix_rows, pos] come from its cache.
 * Requires: no position of the call wraps the ring (pos < window), every
 * listed sequence at pos >= prefix_rows, prefix_seq at pos >= prefix_rows
 * (rows written); else ND_ATTN_ERR_RANGE and nothing is launched. A prefix too
 * large to stage in shared memory, and a call of fewer than 8192 (sequence, KV
 * head) pairs (too few to fill the GPU that way), run as nd_attn_decode; with
 * ND_ATTN_SHARED_VARIANT=2 (or 1) in the environment when the handle is
 * opened, every call that fits uses the shared-prefix kernels (2: the
 * one-lane-per-query-row kernel where built, head dims up to 64; 1: the lane-
 * map kernel). DEVICE pointers. Does not advance. */
ND_ATTN_API int  nd_attn_decode_shared(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids,
                                       uint32_t prefix_seq, uint32_t prefix_rows, const void *q,
                                       const void *k, const void *v, const void *gate, void *out);
/* Causal prefill of len[i] tokens for each of `n` sequences, starting at their
 * current positions: exactly len[i] successive decode steps of the reference
 * (esp32/main/main.c:233-234, host/nd_dump.c:265-271), i.e. token t appends
 * its K/V and attends to the sink run plus the recent run ending at itself.
 * len is a HOST array; tensors are DEVICE pointers. Does not advance. */
ND_ATTN_API int  nd_attn_prefill(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids,
                     const uint32_t *len, const void *q, const void *k, const void *v,
                     const void *gate, void *out);
/* K1 alone: the head norm + RoPE and the KV store of attention()
 * (nd_model.c:2419-2449) without the attention. For len[i] tokens of each
 * listed sequence at positions [pos, pos + len[i]) (its current position; NULL
 * len = one token each; not advanced), k is normed with the layer's k_norm,
 * rotated and stored with v at kv_slot(position), in the handle's cache format
 * (int8: the bytes and scales of kv_store_int8, nd_model.c:1822-1866). q,
 * when not NULL, is normed with q_norm and rotated IN PLACE, as zcrms_heads /
 * apply_rope do to m->q (nd_model.c:326-397), in the reference's statement
 * order: with f32 activations the bits equal the reference's. Tokens of one
 * sequence that land on the same ring slot are stored in position order (the
 * last one stays). With conv taps, q/k/v are the raw projections (convolved
 * first; q receives the convolved, rotated rows). DEVICE pointers; len is a
 * HOST array. */
ND_ATTN_API int  nd_attn_rope_append(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids,
                                     const uint32_t *len, void *q, const void *k, const void *v);
/* Same as nd_attn_decode / nd_attn_prefill with q/k/v/gate/out in HOST memory;
 * both return after the work has completed. This is the form the reference
 * engine's attention() seam calls (its buffers m->q, m->kbuf, m->vbuf,
 * m->gate, m->attn are host floats, nd_model.c:1169-1173).
 * decode_host: buffers that are pinned and mapped (cudaHostAlloc,
 * cudaMallocHost, cudaHostRegister) are read and written in place by the
 * kernels; pageable ones go through the handle's pinned staging with a host
 * copy. No copy-engine transfer is issued. Device memory is refused
 * (ND_ATTN_ERR_ARG).
 * prefill_host: copies in through device staging, runs, copies out. */
ND_ATTN_API int  nd_attn_decode_host(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids,
                         const void *q, const void *k, const void *v, const void *gate,
                         void *out);
ND_ATTN_API int  nd_attn_prefill_host(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids,
                          const uint32_t *len, const void *q, const void *k, const void *v,
                          const void *gate, void *out);

/* ---- allocation-free decode ------------------------------------------------ */
/* No counterpart in the reference engine (which allocates everything at
 * nd_model_open and has no GPU scratch to place).
 *
 * Same work and arguments as nd_attn_decode for sequences 0..n-1 (no seq_ids),
 * for callers that must not let the library allocate device memory after
 * start-up: hosts that hand out all GPU memory from their own fixed budget,
 * and serving loops where a cudaMalloc/cudaFree (which can synchronise the
 * device or fail under fragmentation) is not allowed on the request path.
 * The split-KV partial results and merge tickets live in one fixed array in
 * the library's device image, ND_ATTN_NOALLOC_SCRATCH_BYTES per GPU, held
 * from the first load of the library on that GPU until process exit; this call
 * makes no cudaMalloc/cudaFree and no allocating library call.
 * Limits: n * n_kv_heads <= ND_ATTN_NOALLOC_MAX_ITEMS, else ND_ATTN_ERR_RANGE
 * and nothing is launched; when the partial results of the chosen split would
 * not fit, fewer splits are used (never more memory).
 * The first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture. The
 * address is kept for the life of the process: after cudaDeviceReset (or any
 * other teardown of the device's primary context) this entry point must not be
 * called on that device again.
 * Every call on a device shares the one array: calls that can run at the same
 * time on the GPU (two handles on different streams) race and must be
 * serialised by the caller. The array keeps the previous call's contents; the
 * merge tickets are cleared on the handle's stream at the start of every call
 * that splits (a call without splits does not use them). */
#define ND_ATTN_NOALLOC_SCRATCH_BYTES (8u << 20)
#define ND_ATTN_NOALLOC_MAX_ITEMS     16384u
ND_ATTN_API int  nd_attn_decode_noalloc(nd_attn *h, uint32_t layer, uint32_t n, const void *q,
                                        const void *k, const void *v, const void *gate, void *out);

/* ---- head-sharded decode over several GPUs ---------------------------------- */
/* The reference splits attention by KV group across its two cores
 * (attn_heads' head split, engine/src/nd_model.c:2125-2131); this is the same
 * split across the GPUs of one box, one process (rank) per GPU. Every rank
 * opens its handle with the geometry of ITS heads (n_heads / world query heads,
 * n_kv_heads / world KV heads; rank r owns KV heads [r*n_kv/world,
 * (r+1)*n_kv/world) and their query heads) and holds the same sequences at the
 * same positions. A gathered decode computes the rank's heads and writes each
 * output row straight into every rank's gather buffer (peer stores over
 * NVLink, inside the attention kernel); every rank's `out` then holds all
 * heads, [n][world * n_heads * v_head_dim] of out_dtype, rank r's heads at
 * columns [r * n_heads * v_head_dim, (r + 1) * n_heads * v_head_dim).
 *
 * Set-up, collective over the ranks:
 *  1. nd_attn_gather_init on every rank: allocates the rank's gather buffer
 *     and fills its ND_ATTN_GATHER_BLOB_BYTES record (IPC handle, GPU id,
 *     geometry);
 *  2. the caller exchanges the records by any transport (MPI, a TCP store,
 *     torch.distributed) into an array in rank order;
 *  3. nd_attn_gather_attach on every rank with that array (maps the peers'
 *     buffers), then a barrier across the ranks before the first gathered
 *     decode.
 * nd_attn_gather_check validates such an array on the host alone (no GPU):
 * rank order, equal geometry, one GPU per rank.
 *
 * nd_attn_decode_gather: the arguments of nd_attn_decode (q/k/v/gate of the
 * rank's heads, DEVICE pointers), `out` as above (8-byte aligned). Collective:
 * every rank makes the same sequence of gathered calls with the same n.
 * Returns after enqueueing, like nd_attn_decode. Each 8-byte word a kernel
 * stores into a peer's buffer carries 4 bytes of output and the call's number,
 * so no fence or flag is needed; a bounded device wait (~2 s) for the other
 * ranks' words ends the call, and when it expires nd_attn_sync reports
 * ND_ATTN_ERR_TIMEOUT (a rank that stopped or never made the call). One rank
 * per GPU: the ranks' kernels wait for one another, so two ranks on one GPU
 * are refused. Peers' buffers are released by nd_attn_close, which the ranks
 * call after a final barrier. No counterpart in the reference engine. */
#define ND_ATTN_GATHER_BLOB_BYTES 128u
ND_ATTN_API int  nd_attn_gather_check(const void *records, uint32_t world, uint32_t rank);
ND_ATTN_API int  nd_attn_gather_init(nd_attn *h, uint32_t rank, uint32_t world, void *record);
ND_ATTN_API int  nd_attn_gather_attach(nd_attn *h, const void *records);
ND_ATTN_API int  nd_attn_decode_gather(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids,
                                       const void *q, const void *k, const void *v, const void *gate,
                                       void *out);

/* ---- schema-prefix KV ------------------------------------------------------ */
/* nd_model_prefix_save (nd_model.c:1531-1541): requires a snapshot at the
 * current position; copies the live slots [0, min(snap_pos+1, window)) of
 * every layer into device memory owned by the returned prefix. NULL on error. */
ND_ATTN_API nd_attn_prefix *nd_attn_prefix_save(nd_attn *h, uint32_t seq);
/* nd_model_prefix_restore (nd_model.c:1543-1553): -1 if the prefix belongs to
 * another handle; may target any sequence of the owning handle. */
ND_ATTN_API int  nd_attn_prefix_restore(nd_attn *h, uint32_t seq, const nd_attn_prefix *p);
ND_ATTN_API void nd_attn_prefix_free(nd_attn_prefix *p);
/* Size of the prefix image and, if host != NULL and cap is enough, the image
 * itself in the reference's byte order (prefix_copy, nd_model.c:1493-1529):
 * K rows per layer, V rows per layer, k_scale rows, v_scale rows (scales only
 * with int8 KV). */
ND_ATTN_API int  nd_attn_prefix_read(const nd_attn_prefix *p, void *host, size_t cap, size_t *bytes,
                         uint32_t *pos, uint32_t *n_sink);

/* ---- cache access (tests, bench set-up) ------------------------------------ */
/* Reads `n_slots` slots [slot0, slot0+n_slots) of one (layer, sequence) in the
 * reference layout into HOST buffers: k [n][n_kv_heads*qk_head_dim],
 * v [n][n_kv_heads*v_head_dim] of kv_dtype, scales [n][n_kv_heads] (int8 only;
 * nullable). Slot indices are logical (kv_slot space), paging is resolved. */
ND_ATTN_API int  nd_attn_read_cache(nd_attn *h, uint32_t layer, uint32_t seq, uint32_t slot0,
                        uint32_t n_slots, void *k, void *v, float *k_scale, float *v_scale);
/* Writes the same layout from DEVICE buffers (synthetic contexts). */
ND_ATTN_API int  nd_attn_write_cache(nd_attn *h, uint32_t layer, uint32_t seq, uint32_t slot0,
                         uint32_t n_slots, const void *k, const void *v,
                         const float *k_scale, const float *v_scale);
/* Paged mode: installs the block table of one sequence (HOST array of
 * window/block_size page ids, each < n_blocks). Pages may be shared between
 * sequences (a common schema prefix). */
ND_ATTN_API int  nd_attn_set_block_table(nd_attn *h, uint32_t seq, const int32_t *pages);

/* ---- hook table ------------------------------------------------------------ */
/* The engine's attention() seam calls through a table of function pointers that
 * defaults to its own C path and is swapped at link or run time, the pattern of
 * the nd_parallel_rows hook (engine/include/nd_quant.h:229-230,
 * engine/src/nd_quant.c:717). nd_attn_cuda_ops() returns this library's table;
 * its members are the entry points declared above. No reference counterpart
 * for the accessor itself. */
#define ND_ATTN_OPS_VERSION 2u
typedef struct nd_attn_ops {
    uint32_t version;   /* ND_ATTN_OPS_VERSION */
    int  (*open)(const nd_attn_config *cfg, nd_attn **out);
    void (*close)(nd_attn *h);
    int  (*set_head_norm)(nd_attn *h, uint32_t layer, const float *q_scale, const float *k_scale);
    int  (*reset)(nd_attn *h, uint32_t seq);
    int  (*set_sink)(nd_attn *h, uint32_t seq, uint32_t n);
    int  (*snapshot)(nd_attn *h, uint32_t seq);
    int  (*rewind)(nd_attn *h, uint32_t seq);
    int  (*advance)(nd_attn *h, uint32_t n, const uint32_t *seq_ids, const uint32_t *len);
    int  (*decode)(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const void *q,
                   const void *k, const void *v, const void *gate, void *out);
    int  (*prefill)(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const uint32_t *len,
                    const void *q, const void *k, const void *v, const void *gate, void *out);
    int  (*decode_host)(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids, const void *q,
                        const void *k, const void *v, const void *gate, void *out);
    int  (*prefill_host)(nd_attn *h, uint32_t layer, uint32_t n, const uint32_t *seq_ids,
                         const uint32_t *len, const void *q, const void *k, const void *v,
                         const void *gate, void *out);
    nd_attn_prefix *(*prefix_save)(nd_attn *h, uint32_t seq);
    int  (*prefix_restore)(nd_attn *h, uint32_t seq, const nd_attn_prefix *p);
    void (*prefix_free)(nd_attn_prefix *p);
    int  (*sync)(nd_attn *h);
    const char *(*last_error)(void);
    int  (*set_conv_taps)(nd_attn *h, uint32_t layer, const float *wq, const float *wk, const float *wv);
} nd_attn_ops;
ND_ATTN_API const nd_attn_ops *nd_attn_cuda_ops(void);

/* ---- misc ------------------------------------------------------------------ */
/* Waits for all work enqueued on the handle's stream; reports device-side
 * status (ND_ATTN_ERR_TIMEOUT) and asynchronous CUDA errors. */
ND_ATTN_API int  nd_attn_sync(nd_attn *h);
/* Failure-path self-test: one device thread waits on an mbarrier that nothing
 * arrives on, bounded to about `limit_us` microseconds (1..1000000), then
 * reports the expiry through the device status word as the hot kernels'
 * bounded waits do. Returns what nd_attn_sync() then reports:
 * ND_ATTN_ERR_TIMEOUT when the path works. The handle stays usable. */
ND_ATTN_API int  nd_attn_selftest_wait(nd_attn *h, uint32_t limit_us);
/* The handle's CUDA stream (a cudaStream_t), for callers that order their own
 * work against it. */
ND_ATTN_API void *nd_attn_stream(nd_attn *h);
/* Makes the handle enqueue on `stream` (a cudaStream_t of the handle's device,
 * owned by the caller); NULL goes back to the handle's own stream. */
ND_ATTN_API int  nd_attn_set_stream(nd_attn *h, void *stream);
/* Number of kernels this handle has launched since open. */
ND_ATTN_API uint64_t nd_attn_launch_count(const nd_attn *h);
/* Last error message of the calling thread ("" if none). */
ND_ATTN_API const char *nd_attn_last_error(void);
/* Library build string (arch, version). */
ND_ATTN_API const char *nd_attn_version(void);

#ifdef __cplusplus
}
#endif
#endif /* ND_ATTN_H */
