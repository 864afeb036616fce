/* nd_oracle.c - TEST INFRASTRUCTURE ONLY: the CPU restatement of the Needle
 * attention hot path that the CUDA library is checked against. Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load it.
 *
 * It restates, per token of one (layer, sequence):
 *   - RoPE tables: inv[i] = 1/powf(theta, 2i/hd)  (engine/src/nd_model.c:1233-1236)
 *     and cos/sin((float)pos*inv[i])              (nd_model.c:2949-2954);
 *   - optional per-head ZC-RMSNorm fused with NeoX half-split RoPE
 *     (zcrms_head_rows, nd_model.c:326-365), or pure RoPE (apply_rope,
 *     nd_model.c:381-397), in the reference's fp32 operation order with no
 *     contraction, so the rotated K is bit-identical;
 *   - the KV store at kv_slot(pos) (nd_model.c:1304-1309, 2426-2449): int8 with
 *     scale max|x|/127 (1 if 0) and a correctly rounded quotient, clamp to
 *     +-127, round half to even (kv_store_int8, nd_model.c:1822-1866); or the
 *     value rounded to nearest-even f16/bf16, or kept f32;
 *   - attention over the sink run [0, min(n_sink,pos+1)) and the recent run
 *     ending at pos (nd_model.c:2451-2481) with scores (q.k)*(k_scale/sqrt(qk_hd)),
 *     a running-max softmax, and P.V with v_scale (attn_heads, nd_model.c:2105-2359),
 *     accumulated in double: this is the tolerance reference;
 *   - the emit o/den * sigmoid(gate) (attn_gate_emit, nd_model.c:2091-2103).
 *
 * Build flags must keep -ffp-contract=off: the fp32 RoPE statements are
 * evaluated with separately rounded multiplies and adds, as the reference is
 * when built without FMA contraction.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { NDO_I8 = 0, NDO_F32 = 1, NDO_F16 = 2, NDO_BF16 = 3 };

typedef struct {
    uint32_t n_heads, n_kv_heads, qk_head_dim, v_head_dim, window;
    int32_t  kv_dtype;
} ndo_geom;

/* ---- element conversions (IEEE round to nearest even) ------------------- */
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t ndo_f32_to_bf16(float f)
{
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u)          /* NaN: keep it quiet */
        return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float ndo_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint16_t ndo_f32_to_f16(float f)
{
    uint32_t u = f2u(f), sign = (u >> 16) & 0x8000u, a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);           /* NaN */
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);          /* rounds to inf */
    if (a < 0x38800000u) {                                            /* f16 subnormal/zero */
        /* value = a_float; f16 subnormal unit = 2^-24. */
        uint32_t e = a >> 23, m = (a & 0x7fffffu) | 0x800000u;
        uint32_t shift, q, rem, half;
        if (e < 102u) return (uint16_t)sign;                         /* < 2^-25: rounds to 0 */
        shift = 126u - e;                                            /* m * 2^(e-150) / 2^-24 */
        q = m >> shift;
        rem = m & ((1u << shift) - 1u);
        half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    {
        uint32_t r = a + 0xfffu + ((a >> 13) & 1u);                   /* RNE at bit 13 */
        r -= 0x38000000u;                                            /* rebias 127 -> 15 */
        return (uint16_t)(sign | (r >> 13));
    }
}

float ndo_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) {
        float f = (float)m * 5.9604644775390625e-08f;                /* 2^-24 */
        return sign ? -f : f;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* ---- RoPE ------------------------------------------------------------------ */
void ndo_rope_inv(float theta, uint32_t qk_hd, float *inv)
{
    uint32_t i;
    for (i = 0; i < qk_hd / 2; i++)
        inv[i] = 1.0f / powf(theta, (float)(2 * i) / (float)qk_hd);
}

/* cos/sin table for positions [0, npos): tab[pos][i] = {cos, sin}. */
void ndo_rope_table(float theta, uint32_t qk_hd, uint32_t npos, float *tab)
{
    float    inv[256];
    uint32_t p, i, half = qk_hd / 2;
    ndo_rope_inv(theta, qk_hd, inv);
    for (p = 0; p < npos; p++)
        for (i = 0; i < half; i++) {
            float angle = (float)p * inv[i];
            tab[((size_t)p * half + i) * 2 + 0] = cosf(angle);
            tab[((size_t)p * half + i) * 2 + 1] = sinf(angle);
        }
}

/* In place on `nheads` rows of `dim`: norm (if s) then rotate. */
void ndo_norm_rope(float *x, uint32_t nheads, uint32_t dim, const float *s,
                   const float *cs, const float *sn)
{
    uint32_t h, i, half = dim / 2;
    for (h = 0; h < nheads; h++) {
        float *v = x + (size_t)h * dim;
        if (s) {
            float ss = 0.0f, inv;
            for (i = 0; i < dim; i++) ss = ss + v[i] * v[i];
            inv = 1.0f / sqrtf(ss / (float)dim + 1e-6f);
            for (i = 0; i < half; i++) {
                float x1n = (1.0f + s[i]) * v[i] * inv;
                float x2n = (1.0f + s[i + half]) * v[i + half] * inv;
                v[i]        = x1n * cs[i] - x2n * sn[i];
                v[i + half] = x2n * cs[i] + x1n * sn[i];
            }
            if (half * 2u < dim) v[dim - 1u] = (1.0f + s[dim - 1u]) * v[dim - 1u] * inv;
        } else {
            for (i = 0; i < half; i++) {
                float x1 = v[i], x2 = v[i + half];
                v[i]        = x1 * cs[i] - x2 * sn[i];
                v[i + half] = x2 * cs[i] + x1 * sn[i];
            }
        }
    }
}

/* ---- slots and runs --------------------------------------------------------- */
uint32_t ndo_kv_slot(uint32_t window, uint32_t n_sink, uint32_t p)
{
    return p < n_sink ? p : n_sink + (p - n_sink) % (window - n_sink);
}

uint32_t ndo_set_sink(uint32_t window, uint32_t n)
{
    uint32_t cap = window > 64u ? window - 64u : 0u;
    return n > cap ? cap : n;
}

/* ---- KV store ------------------------------------------------------------------ */
static int8_t ndo_q8(float x, float scale)
{
    float q = x / scale;                  /* correctly rounded, as the residual form is */
    if (q > 127.0f) q = 127.0f;
    if (q < -127.0f) q = -127.0f;
    return (int8_t)lrintf(q);
}

static void ndo_store_row(void *base, int32_t dt, size_t idx, const float *x, uint32_t n,
                          float *scale_out)
{
    uint32_t i;
    switch (dt) {
    case NDO_I8: {
        float mx = 0.0f, sc;
        for (i = 0; i < n; i++) { float a = fabsf(x[i]); if (a > mx) mx = a; }
        sc = mx > 0.0f ? mx / 127.0f : 1.0f;
        *scale_out = sc;
        for (i = 0; i < n; i++) ((int8_t *)base)[idx + i] = ndo_q8(x[i], sc);
        break;
    }
    case NDO_F32:
        for (i = 0; i < n; i++) ((float *)base)[idx + i] = x[i];
        break;
    case NDO_F16:
        for (i = 0; i < n; i++) ((uint16_t *)base)[idx + i] = ndo_f32_to_f16(x[i]);
        break;
    default:
        for (i = 0; i < n; i++) ((uint16_t *)base)[idx + i] = ndo_f32_to_bf16(x[i]);
        break;
    }
}

static double ndo_load(const void *base, int32_t dt, size_t idx)
{
    switch (dt) {
    case NDO_I8:  return (double)((const int8_t *)base)[idx];
    case NDO_F32: return (double)((const float *)base)[idx];
    case NDO_F16: return (double)ndo_f16_to_f32(((const uint16_t *)base)[idx]);
    default:      return (double)ndo_bf16_to_f32(((const uint16_t *)base)[idx]);
    }
}

/* QKV short causal convolution, tap_projection / tap_rows (nd_model.c:
 * 2361-2379, 1753-1802): history slot pos % taps takes the raw row x, then
 *   out[i] = 0 + w[0][i]*h(pos)[i] + w[1][i]*h(pos-1)[i] + ...
 * over min(taps, pos+1) taps in ascending order, every product and sum
 * rounded on its own (no contraction). w and hist are [taps][dim]. */
int ndo_conv_taps(uint32_t taps, uint32_t pos, uint32_t dim, const float *w, const float *x, float *hist,
                  float *out)
{
    uint32_t i, j, nt;

    if (!taps) return -1;
    nt = taps < pos + 1u ? taps : pos + 1u;
    memcpy(hist + (size_t)(pos % taps) * dim, x, (size_t)dim * sizeof(float));
    for (i = 0; i < dim; i++) {
        float acc = 0.0f;
        for (j = 0; j < nt; j++) {
            const float prod = w[(size_t)j * dim + i] * hist[(size_t)((pos - j) % taps) * dim + i];
            acc = acc + prod;
        }
        out[i] = acc;
    }
    return 0;
}


/* Rotate q/k (in place), store k/v at kv_slot(pos), attend. Caches are one
 * (layer, sequence) view: k [window][n_kv*qk_hd], v [window][n_kv*v_hd],
 * scales [window][n_kv] (int8 only). gate NULL = gate of 1. out is double
 * [n_heads][v_hd]. Returns 0, or -1 on bad geometry. */
int ndo_token(const ndo_geom *g, void *k_cache, void *v_cache, float *k_scale,
              float *v_scale, uint32_t pos, uint32_t n_sink, const float *cs,
              const float *sn, const float *qnorm, const float *knorm, float *q,
              float *k, const float *v, const float *gate, double *out)
{
    uint32_t nh = g->n_heads, nkv = g->n_kv_heads, qk = g->qk_head_dim, vh = g->v_head_dim;
    uint32_t W = g->window, rep, slot, kh, h, i, run, sinks, rfirst, rcount;
    size_t   kdim = (size_t)nkv * qk, vdim = (size_t)nkv * vh;
    double   scale;

    if (!nkv || nh % nkv || qk > 256 || vh > 256 || n_sink >= W) return -1;
    rep = nh / nkv;
    ndo_norm_rope(q, nh, qk, qnorm, cs, sn);
    ndo_norm_rope(k, nkv, qk, knorm, cs, sn);

    slot = ndo_kv_slot(W, n_sink, pos);
    for (kh = 0; kh < nkv; kh++) {
        float ks = 1.0f, vs = 1.0f;
        ndo_store_row(k_cache, g->kv_dtype, slot * kdim + (size_t)kh * qk, k + (size_t)kh * qk, qk, &ks);
        ndo_store_row(v_cache, g->kv_dtype, slot * vdim + (size_t)kh * vh, v + (size_t)kh * vh, vh, &vs);
        if (g->kv_dtype == NDO_I8) {
            k_scale[(size_t)slot * nkv + kh] = ks;
            v_scale[(size_t)slot * nkv + kh] = vs;
        }
    }

    sinks = n_sink < pos + 1 ? n_sink : pos + 1;
    if (pos + 1 <= n_sink) { rfirst = pos + 1; rcount = 0; }
    else {
        rcount = pos + 1 - n_sink;
        if (rcount > W - n_sink) rcount = W - n_sink;
        rfirst = pos + 1 - rcount;
    }
    scale = 1.0 / (double)sqrtf((float)qk);

    for (h = 0; h < nh; h++) {
        uint32_t gi = h / rep;
        double   mx = -INFINITY, den = 0.0, acc[256];
        const float *qh = q + (size_t)h * qk;
        for (i = 0; i < vh; i++) acc[i] = 0.0;
        for (run = 0; run < 2; run++) {
            uint32_t base = run ? rfirst : 0, count = run ? rcount : sinks, p;
            for (p = 0; p < count; p++) {
                uint32_t sl = ndo_kv_slot(W, n_sink, base + p);
                size_t   ko = (size_t)sl * kdim + (size_t)gi * qk;
                size_t   vo = (size_t)sl * vdim + (size_t)gi * vh;
                double   ksc = g->kv_dtype == NDO_I8 ? k_scale[(size_t)sl * nkv + gi] : 1.0;
                double   vsc = g->kv_dtype == NDO_I8 ? v_scale[(size_t)sl * nkv + gi] : 1.0;
                double   s = 0.0, w;
                for (i = 0; i < qk; i++) s += (double)qh[i] * ndo_load(k_cache, g->kv_dtype, ko + i);
                s *= ksc * scale;
                if (s > mx) {
                    double r = exp(mx - s);
                    for (i = 0; i < vh; i++) acc[i] *= r;
                    den *= r;
                    mx = s;
                }
                w = exp(s - mx);
                den += w;
                for (i = 0; i < vh; i++) acc[i] += w * vsc * ndo_load(v_cache, g->kv_dtype, vo + i);
            }
        }
        for (i = 0; i < vh; i++) {
            double gsig = 1.0;
            if (gate) gsig = 1.0 / (1.0 + exp(-(double)gate[(size_t)h * vh + i]));
            out[(size_t)h * vh + i] = acc[i] / den * gsig;
        }
    }
    return 0;
}
