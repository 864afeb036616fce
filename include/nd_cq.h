/* nd_cq.h - the Needle attention block's CQ2 projections on B200 (sm_100a):
 * the `.cact` archive reader and the 2-bit Cactus-Quants q/k/v/gate and out
 * projections that feed and drain the attention library (nd_attn.h), as a C
 * ABI in the same shared library (libndattn.so).
 *
 * Reference: the archive reader engine/src/nd_cact.c (format in
 * engine/include/nd_cact.h:1-99) and the projection path of attention()
 * (engine/src/nd_model.c:2402-2411, 2495-2501): nd_cq_prepare (per-group
 * Walsh-Hadamard transform of the activation, scaled by 1/sqrt(group);
 * engine/src/nd_quant.c:354-380), nd_cq_lut_build (16-entry pair table per two
 * reduction positions; nd_quant.c:75-97, 667-678) and the 2-bit row walk
 * nd_lut2_rows_c (nd_quant.c:718-763). The device kernels evaluate the same
 * statements in the same order with explicitly rounded float operations, so
 * a projection's outputs are the reference's bit for bit.
 *
 * Conventions are nd_attn.h's: 0 or a negative code (nd_cact_open's -1..-5
 * for a bad archive), the handle owns its device copies, plain pointers only,
 * work enqueued on a caller-chosen CUDA stream.
 */
#ifndef ND_CQ_H
#define ND_CQ_H

#include <stddef.h>
#include <stdint.h>

#include "nd_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Directory record dtypes (nd_cact.h:28-33). */
#define ND_CQ_DT_FP16 1
#define ND_CQ_DT_FP32 2
#define ND_CQ_DT_CQ   3
#define ND_CQ_DT_RAW  4

/* Header words (nd_cact_header field order, 49 little-endian u32-sized fields;
 * word 48 is rope_theta's f32 bits). */
#define ND_CQ_HEADER_WORDS 49
#define ND_CQ_H_NUM_TENSORS 1
#define ND_CQ_H_D_MODEL     7
#define ND_CQ_H_NUM_HEADS   8
#define ND_CQ_H_NUM_KV      9
#define ND_CQ_H_NUM_LAYERS  10
#define ND_CQ_H_QK_HD       11
#define ND_CQ_H_V_HD        12
#define ND_CQ_H_MAX_SEQ     13
#define ND_CQ_H_QKV_TAPS    19
#define ND_CQ_H_ROPE_THETA  48

/* One decoded directory record (nd_tensor, nd_cact.h:70-79). */
typedef struct {
    uint8_t  dtype, ndim;
    uint32_t shape[4];
    uint64_t offset, nbytes;
    uint32_t group, bits;
} nd_cq_tensor;

typedef struct nd_cq nd_cq;

/* Parses `size` bytes of a .cact archive with nd_cact_open's checks
 * (nd_cact.c:22-76) and keeps a host copy. With device >= 0 it also copies
 * the codebook and every 2-bit CQ tensor to that GPU for nd_cq_project; with
 * device < 0 the handle only reads (no GPU is touched). Returns 0, -1..-5 as
 * nd_cact_open for a bad archive, or ND_ATTN_ERR_NOMEM / ND_ATTN_ERR_CUDA. */
ND_ATTN_API int  nd_cq_open(const void *blob, size_t size, int device, nd_cq **out);
ND_ATTN_API void nd_cq_close(nd_cq *c);

/* The 49 header words. */
ND_ATTN_API int nd_cq_header(const nd_cq *c, uint32_t words[ND_CQ_HEADER_WORDS]);
/* Directory record `index` (nd_cact_tensor, nd_cact.c:91-116): shape words
 * past ndim read as 0. ND_ATTN_ERR_RANGE past the directory. */
ND_ATTN_API int nd_cq_tensor_info(const nd_cq *c, uint32_t index, nd_cq_tensor *t);
/* Directory index of slot `slot` (0..26: norm_in, q_proj, k_proj, v_proj,
 * q/k/v_taps, q_norm, k_norm, gate_proj, out_proj, ...) of layer `layer`:
 * 1 + layer * (taps ? 27 : 24) + slot (bind_layer, nd_model.c:642-658). */
ND_ATTN_API int nd_cq_layer_tensor(const nd_cq *c, uint32_t layer, uint32_t slot, uint32_t *index);
/* An FP16 or FP32 tensor's elements as host floats (nd_f16 for halves);
 * `cap` floats of room. ND_ATTN_ERR_ARG for other dtypes or too little room. */
ND_ATTN_API int nd_cq_read_f32(const nd_cq *c, uint32_t index, float *host, size_t cap);

/* y_i = W_i x for n_tensors CQ2 tensors that reduce over the same input
 * (equal shape[1] and group, as q/k/v/gate in attention()): one prepare and
 * one pair table per token serve them all. x: device [n_tok][shape[1]] f32;
 * y[i]: device [n_tok][shape[0] of tensor i] f32. Enqueued on `stream` (a
 * cudaStream_t of the handle's device; NULL = the legacy default stream).
 * Limits: at most 8 tensors per call, 2-bit tensors, group a power of two from
 * 16 to 256, padded input <= 4096. */
ND_ATTN_API int nd_cq_project(nd_cq *c, uint32_t n_tensors, const uint32_t *tensors, uint32_t n_tok,
                              const float *x, float *const *y, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* ND_CQ_H */
