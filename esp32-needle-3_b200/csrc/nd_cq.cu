// nd_cq.cu - the Needle attention block's CQ2 projections on sm_100a, and the
// `.cact` archive reader behind them (include/nd_cq.h).
//
// A CQ2 tensor W [out][in] holds, per row, 2-bit codebook indices (an
// LSB-first bit stream, in padded to a multiple of the group g) and an f16
// norm per group. The reference computes y = W x as (nd_quant.c):
//   xh  = per group of g: Walsh-Hadamard transform of x (zero-padded), times
//         1/sqrt(g)                                   nd_cq_prepare  354-380
//   T   = per pair p of reduction positions, 16 entries
//         T[p][i0 + 4 i1] = cb[i0] xh[2p] + cb[i1] xh[2p+1]
//                                                      lutb_rows 75-97 (build 667-678)
//   y_r = sum over groups of f16(norm) * ((s0 + s1) + (s2 + s3)), s_k the
//         running sums of the table entries that the k-th nibble of each 16-bit
//         half-word of the row's index words selects   nd_lut2_rows_c 722-763
// The kernel below evaluates exactly these statements in this order, with
// explicitly rounded float operations (no contraction into FMAs: the
// reference's engine build has none on its target and the checker is built
// with -ffp-contract=off), so the outputs are the reference's bit for bit.
//
// One launch per call (cq_project_kernel): a CTA takes 128 output rows of one
// of the call's tensors for TT tokens, rebuilds those tokens' transforms and
// pair tables in shared memory (cheap next to the row walks, and no table
// round trip through global memory), then every thread walks its row's index
// words once for all TT tokens. The projections of the attention block are
// small (the reference model's q/k/v/gate/out are 768 x 768 at most, 2 bits
// per weight): work per call is a few microseconds of table lookups, not
// tensor-core shaped.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/nd_cq.h"
#include "nd_internal.h"

namespace {

constexpr uint32_t kHeaderWords = ND_CQ_HEADER_WORDS;
constexpr uint32_t kHeaderBytes = kHeaderWords * 4;
constexpr uint32_t kRecordBytes = 44;
constexpr uint32_t kTag = 0x05E12A84u;
constexpr uint32_t kMaxInPad = 4096;   // one token's table and transform: in_pad * 36 bytes of shared memory
constexpr size_t kSmemBudget = 112 * 1024;   // two CTAs per SM where TT allows
constexpr int kRowsPerCta = 128;

uint32_t rd_u32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
uint64_t rd_u64(const uint8_t *p) { return (uint64_t)rd_u32(p) | ((uint64_t)rd_u32(p + 4) << 32); }

// nd_f16 (nd_quant.h:50): exact half -> float, subnormals included.
float half_bits_to_float(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

// The tensors of one nd_cq_project call, each a run of 128-row blocks of the
// grid's x dimension.
constexpr int kMaxJobs = 8;
struct CqJob {
    const uint8_t *packed;     // [out][rowbytes] indices
    const uint16_t *norms;     // [out][ngroup] f16
    float *y;                  // [n_tok][out]
    uint32_t out, rb0;         // rows, first row block
};
struct CqJobs {
    CqJob job[kMaxJobs];
    uint32_t n;
};

// One CTA of 128 x TT threads: 128 output rows of one tensor for TT tokens.
// Phase 1 stages the tokens' activations, runs the per-group butterflies
// (every butterfly of a stage in parallel: each element's sequence of adds is
// the reference's whatever the order), scales, and builds the tokens' pair
// tables in shared memory. Phase 2: thread (row, token) walks the row's index
// words and norms and accumulates in the reference's order (per group the
// four running sums, then acc += f16(norm) * ((s0 + s1) + (s2 + s3))).
template <int TT>
__global__ void __launch_bounds__(kRowsPerCta * 4) cq_project_kernel(const float *__restrict__ x, uint32_t n_tok,
                                                                 uint32_t in, uint32_t in_pad, uint32_t g, float scale,
                                                                 float4 cb, const __grid_constant__ CqJobs jobs) {
    extern __shared__ float4 smem4[];
    float *lut = reinterpret_cast<float *>(smem4);          // [TT][in_pad / 2][16]
    float *xh = lut + (size_t)TT * in_pad * 8;               // [TT][in_pad]
    const uint32_t tid = threadIdx.x, nt = blockDim.x, t0 = blockIdx.y * TT;
    const uint32_t ntt = min((uint32_t)TT, n_tok - t0);
#pragma unroll
    for (int tt = 0; tt < TT; tt++)
        for (uint32_t c = tid; c < in_pad; c += nt)
            xh[(size_t)tt * in_pad + c] = (uint32_t)tt < ntt && c < in ? x[(size_t)(t0 + tt) * in + c] : 0.0f;
    __syncthreads();
    // nd_fwht (nd_quant.c:20-58): stages len = 1, 2, .., g/2; butterfly
    // (j, j + len) of a block of 2 len within a group becomes (a + b, a - b).
    // g is a power of two: butterfly b of a token sits in group b >> lg_h at
    // (k >> ls) << (ls + 1) | (k & (len - 1)), k = b & (g/2 - 1).
    const uint32_t half_g = g / 2, npairs = in_pad / 2, lg_h = __ffs(half_g) - 1;
    for (uint32_t ls = 0, len = 1; len < g; ls++, len <<= 1) {
#pragma unroll
        for (int tt = 0; tt < TT; tt++) {
            float *xt = xh + (size_t)tt * in_pad;
            for (uint32_t b = tid; b < npairs; b += nt) {
                const uint32_t k = b & (half_g - 1);
                float *blk = xt + ((b >> lg_h) << (lg_h + 1)) + ((k >> ls) << (ls + 1)) + (k & (len - 1));
                const float a = blk[0], c = blk[len];
                blk[0] = __fadd_rn(a, c);
                blk[len] = __fsub_rn(a, c);
            }
        }
        __syncthreads();
    }
    // fw_scale (nd_quant.c:99-110), then the pair table (lutb_rows, 75-97):
    // T[i0 + 4 i1] = cb[i0] x0 + cb[i1] x1.
#pragma unroll
    for (int tt = 0; tt < TT; tt++)
    for (uint32_t p = tid; p < npairs; p += nt) {
        const float x0 = __fmul_rn(xh[(size_t)tt * in_pad + 2 * p], scale);
        const float x1 = __fmul_rn(xh[(size_t)tt * in_pad + 2 * p + 1], scale);
        const float a0 = __fmul_rn(cb.x, x0), a1 = __fmul_rn(cb.y, x0), a2 = __fmul_rn(cb.z, x0),
                    a3 = __fmul_rn(cb.w, x0);
        const float b0 = __fmul_rn(cb.x, x1), b1 = __fmul_rn(cb.y, x1), b2 = __fmul_rn(cb.z, x1),
                    b3 = __fmul_rn(cb.w, x1);
        float4 *T4 = reinterpret_cast<float4 *>(lut + ((size_t)tt * npairs + p) * 16);
        T4[0] = make_float4(__fadd_rn(a0, b0), __fadd_rn(a1, b0), __fadd_rn(a2, b0), __fadd_rn(a3, b0));
        T4[1] = make_float4(__fadd_rn(a0, b1), __fadd_rn(a1, b1), __fadd_rn(a2, b1), __fadd_rn(a3, b1));
        T4[2] = make_float4(__fadd_rn(a0, b2), __fadd_rn(a1, b2), __fadd_rn(a2, b2), __fadd_rn(a3, b2));
        T4[3] = make_float4(__fadd_rn(a0, b3), __fadd_rn(a1, b3), __fadd_rn(a2, b3), __fadd_rn(a3, b3));
    }
    __syncthreads();
    // Thread (row, token): which tensor's block this is, then the row's index
    // words and norms, the next group's fetched while this one is summed.
    uint32_t j = 0;
    while (j + 1 < jobs.n && blockIdx.x >= jobs.job[j + 1].rb0) j++;
    const CqJob &J = jobs.job[j];
    const uint32_t r = (blockIdx.x - J.rb0) * kRowsPerCta + tid % kRowsPerCta, tt = tid / kRowsPerCta;
    if (r >= J.out || tt >= ntt) return;
    const uint32_t ngroup = in_pad / g, wpg = g / 16;   // index words per group
    const uint32_t *row = reinterpret_cast<const uint32_t *>(J.packed + (size_t)r * (in_pad / 4));
    const uint16_t *nrm = J.norms + (size_t)r * ngroup;
    const float *Tt = lut + (size_t)tt * npairs * 16;
    uint32_t wv[16], wn[16];   // g <= 256
    uint16_t hn = nrm[0];
#pragma unroll
    for (uint32_t q = 0; q < 16; q++) wv[q] = q < wpg ? row[q] : 0u;
    float acc = 0.0f;
    for (uint32_t gi = 0; gi < ngroup; gi++) {
        const bool more = gi + 1 < ngroup;
        const uint16_t hnext = more ? nrm[gi + 1] : (uint16_t)0;
#pragma unroll
        for (uint32_t q = 0; q < 16; q++) wn[q] = more && q < wpg ? row[(gi + 1) * wpg + q] : 0u;
        __half_raw hr;
        hr.x = hn;
        const float nf = __half2float(__half(hr));
        const float *T = Tt + (size_t)gi * half_g * 16;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
#pragma unroll
        for (uint32_t q = 0; q < 16; q++) {
            if (q < wpg) {
                const uint32_t w = wv[q];
                s0 = __fadd_rn(s0, T[w & 15u]);
                s1 = __fadd_rn(s1, T[16 + ((w >> 4) & 15u)]);
                s2 = __fadd_rn(s2, T[32 + ((w >> 8) & 15u)]);
                s3 = __fadd_rn(s3, T[48 + ((w >> 12) & 15u)]);
                s0 = __fadd_rn(s0, T[64 + ((w >> 16) & 15u)]);
                s1 = __fadd_rn(s1, T[80 + ((w >> 20) & 15u)]);
                s2 = __fadd_rn(s2, T[96 + ((w >> 24) & 15u)]);
                s3 = __fadd_rn(s3, T[112 + (w >> 28)]);
                T += 128;
            }
        }
        acc = __fadd_rn(acc, __fmul_rn(nf, __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3))));
        hn = hnext;
#pragma unroll
        for (uint32_t q = 0; q < 16; q++) wv[q] = wn[q];
    }
    J.y[(size_t)(t0 + tt) * J.out + r] = acc;
}

}  // namespace

struct nd_cq {
    std::vector<uint8_t> blob;      // host copy of the archive
    uint32_t hdr[kHeaderWords];
    size_t dir_off = 0;
    uint32_t n = 0;
    int device = -1;
    uint8_t *d_blob = nullptr;      // device copy (CQ tensors and codebook read in place)
};

namespace {

void decode_record(const nd_cq *c, uint32_t i, nd_cq_tensor *t) {
    const uint8_t *r = c->blob.data() + c->dir_off + (size_t)i * kRecordBytes;
    t->dtype = r[0];
    t->ndim = r[1];
    for (int d = 0; d < 4; d++) t->shape[d] = d < t->ndim ? rd_u32(r + 4 + 4 * d) : 0u;
    t->offset = rd_u64(r + 20);
    t->nbytes = rd_u64(r + 28);
    t->group = rd_u32(r + 36);
    t->bits = rd_u32(r + 40);
}

bool in_blob(const nd_cq *c, const nd_cq_tensor &t) {
    return t.offset <= c->blob.size() && t.nbytes <= c->blob.size() - t.offset;
}

// Checks a tensor nd_cq_project can take; fills its padded input and row bytes.
int cq2_geometry(const nd_cq *c, uint32_t index, nd_cq_tensor *t, uint32_t *in_pad, uint32_t *rowbytes) {
    if (index >= c->n) return nda::report_error(ND_ATTN_ERR_RANGE, "tensor %u of %u", index, c->n);
    decode_record(c, index, t);
    if (t->dtype != ND_CQ_DT_CQ || t->bits != 2 || t->ndim != 2)
        return nda::report_error(ND_ATTN_ERR_ARG, "tensor %u is not a 2-bit CQ matrix", index);
    if (t->group < 16 || t->group > 256 || (t->group & (t->group - 1)) || t->shape[0] == 0 || t->shape[1] == 0)
        return nda::report_error(ND_ATTN_ERR_ARG, "tensor %u: group %u", index, t->group);
    *in_pad = (t->shape[1] + t->group - 1) / t->group * t->group;
    *rowbytes = *in_pad / 4;
    const uint64_t need = (uint64_t)t->shape[0] * *rowbytes + (uint64_t)t->shape[0] * (*in_pad / t->group) * 2;
    if (*in_pad > kMaxInPad) return nda::report_error(ND_ATTN_ERR_GEOM, "tensor %u: input %u", index, t->shape[1]);
    if (!in_blob(c, *t) || t->nbytes < need || t->offset % 4 != 0)
        return nda::report_error(ND_ATTN_ERR_ARG, "tensor %u runs past the archive", index);
    return ND_ATTN_OK;
}

}  // namespace

extern "C" {

int nd_cq_open(const void *blob, size_t size, int device, nd_cq **out) {
    if (!out) return nda::report_error(ND_ATTN_ERR_ARG, "null handle pointer");
    *out = nullptr;
    const uint8_t *b = static_cast<const uint8_t *>(blob);
    // nd_cact_open (nd_cact.c:22-76): header, geometry checks, codebook and
    // directory inside the blob.
    if (!b || size < kHeaderBytes) return nda::report_error(-1, "archive shorter than its header");
    uint32_t h[kHeaderWords];
    for (uint32_t i = 0; i < kHeaderWords; i++) h[i] = rd_u32(b + 4 * i);
    if (h[0] != kTag) return nda::report_error(-2, "not a .cact archive (tag %08x)", h[0]);
    const uint32_t d_model = h[7], heads = h[8], kv = h[9], layers = h[10], qk = h[11], vd = h[12];
    const uint32_t hada_n = h[14], num_orders = h[26], num_sites = h[31];
    if (d_model == 0 || layers == 0 || heads == 0 || kv == 0 || qk == 0 || vd == 0 || heads % kv != 0 ||
        heads * vd != d_model || num_orders > 4 || num_sites > 16 || hada_n < d_model)
        return nda::report_error(-3, "archive geometry outside what the engine implements");
    const size_t cb_len = (size_t)h[2] * 4, dir_off = kHeaderBytes + cb_len, dir_len = (size_t)h[1] * kRecordBytes;
    if (dir_off + dir_len < dir_off || dir_off + dir_len > size)
        return nda::report_error(-4, "directory runs past the archive");
    if (h[2] < 28) return nda::report_error(-5, "codebook of %u entries (cb2|cb3|cb4 needs 28)", h[2]);
    nd_cq *c = new (std::nothrow) nd_cq();
    if (!c) return nda::report_error(ND_ATTN_ERR_NOMEM, "handle allocation");
    c->blob.assign(b, b + size);
    memcpy(c->hdr, h, sizeof(h));
    c->dir_off = dir_off;
    c->n = h[1];
    c->device = device;
    if (device >= 0) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaError_t e = cudaSetDevice(device);
        if (e == cudaSuccess) e = cudaMalloc(&c->d_blob, size);
        if (e == cudaSuccess) e = cudaMemcpy(c->d_blob, b, size, cudaMemcpyHostToDevice);
        cudaSetDevice(prev);
        if (e != cudaSuccess) {
            const int code = e == cudaErrorMemoryAllocation ? ND_ATTN_ERR_NOMEM : ND_ATTN_ERR_CUDA;
            nd_cq_close(c);
            return nda::report_error(code, "archive upload: %s", cudaGetErrorString(e));
        }
    }
    *out = c;
    return ND_ATTN_OK;
}

void nd_cq_close(nd_cq *c) {
    if (!c) return;
    if (c->device >= 0) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(c->device);
        cudaFree(c->d_blob);
        cudaSetDevice(prev);
    }
    delete c;
}

int nd_cq_header(const nd_cq *c, uint32_t words[ND_CQ_HEADER_WORDS]) {
    if (!c || !words) return nda::report_error(ND_ATTN_ERR_ARG, "null argument");
    memcpy(words, c->hdr, sizeof(c->hdr));
    return ND_ATTN_OK;
}

int nd_cq_tensor_info(const nd_cq *c, uint32_t index, nd_cq_tensor *t) {
    if (!c || !t) return nda::report_error(ND_ATTN_ERR_ARG, "null argument");
    if (index >= c->n) return nda::report_error(ND_ATTN_ERR_RANGE, "tensor %u of %u", index, c->n);
    decode_record(c, index, t);
    return ND_ATTN_OK;
}

int nd_cq_layer_tensor(const nd_cq *c, uint32_t layer, uint32_t slot, uint32_t *index) {
    if (!c || !index) return nda::report_error(ND_ATTN_ERR_ARG, "null argument");
    const uint32_t per = c->hdr[ND_CQ_H_QKV_TAPS] ? 27u : 24u;
    if (layer >= c->hdr[ND_CQ_H_NUM_LAYERS] || slot >= per)
        return nda::report_error(ND_ATTN_ERR_RANGE, "layer %u slot %u", layer, slot);
    const uint64_t i = 1 + (uint64_t)layer * per + slot;
    if (i >= c->n) return nda::report_error(ND_ATTN_ERR_RANGE, "tensor %llu of %u", (unsigned long long)i, c->n);
    *index = (uint32_t)i;
    return ND_ATTN_OK;
}

int nd_cq_read_f32(const nd_cq *c, uint32_t index, float *host, size_t cap) {
    if (!c || !host) return nda::report_error(ND_ATTN_ERR_ARG, "null argument");
    if (index >= c->n) return nda::report_error(ND_ATTN_ERR_RANGE, "tensor %u of %u", index, c->n);
    nd_cq_tensor t;
    decode_record(c, index, &t);
    if (!in_blob(c, t)) return nda::report_error(ND_ATTN_ERR_ARG, "tensor %u runs past the archive", index);
    const uint8_t *p = c->blob.data() + t.offset;
    if (t.dtype == ND_CQ_DT_FP16) {
        const size_t n = t.nbytes / 2;
        if (cap < n) return nda::report_error(ND_ATTN_ERR_ARG, "%zu floats of room for %zu", cap, n);
        for (size_t i = 0; i < n; i++) host[i] = half_bits_to_float((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8)));
        return ND_ATTN_OK;
    }
    if (t.dtype == ND_CQ_DT_FP32) {
        const size_t n = t.nbytes / 4;
        if (cap < n) return nda::report_error(ND_ATTN_ERR_ARG, "%zu floats of room for %zu", cap, n);
        memcpy(host, p, n * 4);
        return ND_ATTN_OK;
    }
    return nda::report_error(ND_ATTN_ERR_ARG, "tensor %u is neither FP16 nor FP32", index);
}

int nd_cq_project(nd_cq *c, uint32_t n_tensors, const uint32_t *tensors, uint32_t n_tok, const float *x,
                  float *const *y, void *stream) {
    if (!c || !tensors || !y || (n_tok && !x)) return nda::report_error(ND_ATTN_ERR_ARG, "null argument");
    if (c->device < 0 || !c->d_blob) return nda::report_error(ND_ATTN_ERR_ARG, "handle opened without a device");
    if (n_tensors == 0 || n_tok == 0) return ND_ATTN_OK;
    std::vector<nd_cq_tensor> ts(n_tensors);
    if (n_tensors > (uint32_t)kMaxJobs) return nda::report_error(ND_ATTN_ERR_RANGE, "%u tensors per call", n_tensors);
    uint32_t in_pad = 0, in = 0, g = 0;
    for (uint32_t i = 0; i < n_tensors; i++) {
        uint32_t ip = 0, rb = 0;
        int rc = cq2_geometry(c, tensors[i], &ts[i], &ip, &rb);
        if (rc) return rc;
        if (!y[i]) return nda::report_error(ND_ATTN_ERR_ARG, "null output %u", i);
        if (i == 0) in_pad = ip, in = ts[i].shape[1], g = ts[i].group;
        else if (ts[i].shape[1] != in || ts[i].group != g)
            return nda::report_error(ND_ATTN_ERR_ARG, "tensors reduce over different inputs");
    }
    CqJobs jobs;
    memset(&jobs, 0, sizeof(jobs));
    uint32_t blocks = 0;
    for (uint32_t i = 0; i < n_tensors; i++) {
        const uint32_t out = ts[i].shape[0];
        const uint8_t *packed = c->d_blob + ts[i].offset;
        jobs.job[i] = CqJob{packed, reinterpret_cast<const uint16_t *>(packed + (size_t)out * (in_pad / 4)), y[i], out,
                            blocks};
        blocks += (out + kRowsPerCta - 1) / kRowsPerCta;
    }
    jobs.n = n_tensors;
    const size_t per_tok = (size_t)in_pad * 36;   // table (8 floats per input) + transform (1)
    const int tt = per_tok * 4 <= kSmemBudget ? 4 : per_tok * 2 <= kSmemBudget ? 2 : 1;
    const size_t smem = per_tok * tt;
    // The 2-bit slice of the codebook is its first 4 floats (nd_cact_codebook).
    float4 cb;
    memcpy(&cb, c->blob.data() + kHeaderBytes, sizeof(cb));
    const float scale = 1.0f / sqrtf((float)g);   // nd_cq_prepare's scale
    const dim3 grid(blocks, (n_tok + tt - 1) / tt);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != c->device) cudaSetDevice(c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto go = [&](auto kern) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) {
            kern<<<grid, kRowsPerCta * tt, smem, s>>>(x, n_tok, in, in_pad, g, scale, cb, jobs);
            e = cudaGetLastError();
        }
        return e;
    };
    const cudaError_t e = tt == 4 ? go(cq_project_kernel<4>) : tt == 2 ? go(cq_project_kernel<2>) : go(cq_project_kernel<1>);
    const int rc = e == cudaSuccess ? ND_ATTN_OK
                                    : nda::report_error(ND_ATTN_ERR_CUDA, "projection launch: %s", cudaGetErrorString(e));
    if (prev != c->device) cudaSetDevice(prev);
    return rc;
}

}  // extern "C"
