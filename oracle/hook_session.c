/* hook_session.c - TEST INFRASTRUCTURE ONLY: the reference engine's attention()
 * with the library installed through the hook that oracle/nd_attn_hook.patch
 * adds (nd_attn_hook / nd_attn_hook_ctx, after the QKV taps), against the same
 * attention() on its stock C path.
 *
 * Built by oracle/Makefile (target `hook`) from the PATCHED reference sources
 * (copied to _ref/patched/ and patched there; nothing of the reference is kept
 * in this repository), with this file including engine/src/nd_model.c so its
 * static attention() and bind_layer() are in reach, as ndref_harness.c does.
 *
 * Usage: hook_session <archive.cact> <libndattn.so> <tokens> <window> <n_sink>
 *
 * One sequence of `tokens` positions on layer 0 of the archive: each position
 * runs the reference's attention() twice on identical inputs - once with
 * nd_attn_hook NULL (norm + RoPE, int8 KV store and attn_heads in C), once with
 * the hook calling the library's nd_attn_decode_host through nd_attn_cuda_ops()
 * (the run-time swap-in INTEGRATION describes), then nd_attn_advance. It
 * checks the library's int8 K/V bytes and scales against the C caches bit for
 * bit, and each position's attention() output within 1e-3 * max(1, |ref|).
 * Prints one summary line; exit status 0 when everything holds.
 */
#include <dlfcn.h>
#include <stdio.h>
#include <stdlib.h>

#include "nd_attn.h"
#include "nd_model.h"
#include "nd_model.c"

static const nd_attn_ops *g_ops;

/* The hook body INTEGRATION gives for a single-sequence engine. */
static int cuda_attention(void *ctx, uint32_t layer, const float *q, const float *k, const float *v,
                          const float *gate, float *out)
{
    return g_ops->decode_host((nd_attn *)ctx, layer, 1, NULL, q, k, v, gate, out);
}

typedef struct {
    nd_model m;
    nd_layer L;
    float   *inv, *cs, *sn;
} view;

/* The model state attention() reads, as nd_model_open leaves it for layer 0
 * (geometry, bind_layer, fp16 slots through nd_f16, scratch, caches, tap
 * histories) - the set ndref_attention_layer builds. */
static int view_open(view *w, const uint8_t *blob, size_t size, uint32_t window, uint32_t n_sink)
{
    static const int F16[] = { 4, 5, 6, 7, 8 };
    nd_model *m = &w->m;
    uint32_t  k, i, in_pad = 0, taps;
    memset(w, 0, sizeof(*w));
    if (nd_cact_open(&m->c, blob, size) != 0) return -1;
    m->d_model = m->c.h.d_model; m->n_layers = 1;
    m->n_heads = m->c.h.num_heads; m->n_kv_heads = m->c.h.num_kv_heads;
    m->qk_head_dim = m->c.h.qk_head_dim; m->v_head_dim = m->c.h.v_head_dim;
    m->attn_dim = m->n_heads * m->v_head_dim;
    m->k_dim = m->n_kv_heads * m->qk_head_dim; m->v_dim = m->n_kv_heads * m->v_head_dim;
    m->window = window; m->n_sink = n_sink;
    taps = m->c.h.qkv_conv_taps;
    if (!taps) return -2;
    m->layer = &w->L;
    bind_layer(m, 0);
    {
        const nd_tensor *proj[5] = { &w->L.q_proj, &w->L.k_proj, &w->L.v_proj, &w->L.gate_proj, &w->L.out_proj };
        for (i = 0; i < 5; i++)
            if (nd_cq_in_pad(proj[i]) > in_pad) in_pad = nd_cq_in_pad(proj[i]);
    }
    for (k = 0; k < 5; k++) {
        nd_tensor       t;
        const uint16_t *h;
        nd_cact_tensor(&m->c, 1 + F16[k], &t);
        h = (const uint16_t *)nd_cact_data(&m->c, &t);
        m->fp16_slot[0][F16[k]] = (float *)calloc(t.nbytes / 2 + 1, sizeof(float));
        if (!h || !m->fp16_slot[0][F16[k]]) return -12;
        for (i = 0; i < t.nbytes / 2; i++) m->fp16_slot[0][F16[k]][i] = nd_f16(h[i]);
    }
    m->xh = (float *)calloc(in_pad, sizeof(float));
    m->lut = (float *)calloc(nd_cq_lut_floats(in_pad), sizeof(float));
    m->q = (float *)calloc(m->n_heads * m->qk_head_dim, sizeof(float));
    m->kbuf = (float *)calloc(m->k_dim, sizeof(float));
    m->vbuf = (float *)calloc(m->v_dim, sizeof(float));
    m->gate = (float *)calloc(m->attn_dim, sizeof(float));
    m->attn = (float *)calloc(m->attn_dim, sizeof(float));
    m->k_cache = (int8_t *)calloc((size_t)window * m->k_dim, 1);
    m->v_cache = (int8_t *)calloc((size_t)window * m->v_dim, 1);
    m->k_scale = (float *)calloc((size_t)window * m->n_kv_heads, sizeof(float));
    m->v_scale = (float *)calloc((size_t)window * m->n_kv_heads, sizeof(float));
    m->q_hist = (float *)calloc((size_t)taps * m->n_heads * m->qk_head_dim, sizeof(float));
    m->k_hist = (float *)calloc((size_t)taps * m->k_dim, sizeof(float));
    m->v_hist = (float *)calloc((size_t)taps * m->v_dim, sizeof(float));
    w->inv = (float *)calloc(m->qk_head_dim / 2, sizeof(float));
    w->cs = (float *)calloc(m->qk_head_dim / 2, sizeof(float));
    w->sn = (float *)calloc(m->qk_head_dim / 2, sizeof(float));
    if (!m->xh || !m->lut || !m->q || !m->kbuf || !m->vbuf || !m->gate || !m->attn || !m->k_cache ||
        !m->v_cache || !m->k_scale || !m->v_scale || !m->q_hist || !m->k_hist || !m->v_hist || !w->inv ||
        !w->cs || !w->sn)
        return -12;
    /* nd_model_open's rope_inv (nd_model.c:1233-1236). */
    for (i = 0; i < m->qk_head_dim / 2; i++)
        w->inv[i] = 1.0f / powf(m->c.h.rope_theta, (float)(2 * i) / (float)m->qk_head_dim);
    m->rope_cos = w->cs; m->rope_sin = w->sn;
    return 0;
}

/* nd_model_step_hidden's per-position table (nd_model.c:2949-2954). */
static void view_at(view *w, uint32_t pos)
{
    uint32_t i;
    w->m.pos = pos;
    for (i = 0; i < w->m.qk_head_dim / 2; i++) {
        float angle = (float)pos * w->inv[i];
        w->cs[i] = cosf(angle);
        w->sn[i] = sinf(angle);
    }
}

int main(int argc, char **argv)
{
    FILE          *f;
    uint8_t       *blob;
    long           size;
    uint32_t       tokens, window, n_sink, pos, i;
    view           a, b;
    nd_attn       *h = NULL;
    nd_attn_config cfg;
    void          *lib;
    void (*config_init)(nd_attn_config *);
    int  (*read_cache)(nd_attn *, uint32_t, uint32_t, uint32_t, uint32_t, void *, void *, float *, float *);
    const nd_attn_ops *(*get_ops)(void);
    double         worst = 0.0;
    uint64_t       rng = 0x9E3779B97F4A7C15ull;
    int            bad = 0;

    if (argc != 6) {
        fprintf(stderr, "usage: %s archive.cact libndattn.so tokens window n_sink\n", argv[0]);
        return 2;
    }
    tokens = (uint32_t)atoi(argv[3]); window = (uint32_t)atoi(argv[4]); n_sink = (uint32_t)atoi(argv[5]);
    f = fopen(argv[1], "rb");
    if (!f) { perror(argv[1]); return 2; }
    fseek(f, 0, SEEK_END); size = ftell(f); fseek(f, 0, SEEK_SET);
    blob = (uint8_t *)malloc((size_t)size);
    if (!blob || fread(blob, 1, (size_t)size, f) != (size_t)size) { fclose(f); return 2; }
    fclose(f);
    if (view_open(&a, blob, (size_t)size, window, n_sink) || view_open(&b, blob, (size_t)size, window, n_sink)) {
        fprintf(stderr, "archive view failed\n");
        return 2;
    }

    lib = dlopen(argv[2], RTLD_NOW | RTLD_LOCAL);
    if (!lib) { fprintf(stderr, "dlopen: %s\n", dlerror()); return 2; }
    get_ops = (const nd_attn_ops *(*)(void))dlsym(lib, "nd_attn_cuda_ops");
    config_init = (void (*)(nd_attn_config *))dlsym(lib, "nd_attn_config_init");
    read_cache = (int (*)(nd_attn *, uint32_t, uint32_t, uint32_t, uint32_t, void *, void *, float *, float *))
        dlsym(lib, "nd_attn_read_cache");
    if (!get_ops || !config_init || !read_cache) { fprintf(stderr, "missing symbols\n"); return 2; }
    g_ops = get_ops();
    if (!g_ops || g_ops->version != ND_ATTN_OPS_VERSION) { fprintf(stderr, "ops table version\n"); return 2; }
    config_init(&cfg);
    cfg.n_layers = 1; cfg.n_heads = a.m.n_heads; cfg.n_kv_heads = a.m.n_kv_heads;
    cfg.qk_head_dim = a.m.qk_head_dim; cfg.v_head_dim = a.m.v_head_dim;
    cfg.window = window; cfg.max_seqs = 1; cfg.max_pos = window > tokens ? window : tokens;
    cfg.rope_theta = a.m.c.h.rope_theta;
    cfg.kv_dtype = ND_DT_I8; cfg.act_dtype = ND_DT_F32; cfg.out_dtype = ND_DT_F32;
    if (g_ops->open(&cfg, &h) != 0) { fprintf(stderr, "open: %s\n", g_ops->last_error()); return 3; }
    if (g_ops->set_head_norm(h, 0, a.m.fp16_slot[0][7], a.m.fp16_slot[0][8]) != 0 ||
        (n_sink && g_ops->set_sink(h, 0, n_sink) != 0)) {
        fprintf(stderr, "setup: %s\n", g_ops->last_error());
        return 3;
    }

    for (pos = 0; pos < tokens; pos++) {
        float *x = (float *)malloc(sizeof(float) * a.m.d_model);
        float *oa = (float *)malloc(sizeof(float) * a.m.d_model);
        float *ob = (float *)malloc(sizeof(float) * a.m.d_model);
        for (i = 0; i < a.m.d_model; i++) {   /* uniform in [-1.5, 1.5) from a 64-bit LCG */
            rng = rng * 6364136223846793005ull + 1442695040888963407ull;
            x[i] = 3.0f * (float)((rng >> 40) & 0xFFFFFFu) / 16777216.0f - 1.5f;
        }
        view_at(&a, pos);
        view_at(&b, pos);
        nd_attn_hook = NULL;
        nd_attn_hook_ctx = NULL;
        attention(&a.m, 0, x, oa);
        nd_attn_hook = cuda_attention;
        nd_attn_hook_ctx = h;
        attention(&b.m, 0, x, ob);
        nd_attn_hook = NULL;
        if (g_ops->advance(h, 1, NULL, NULL) != 0) { fprintf(stderr, "advance: %s\n", g_ops->last_error()); return 3; }
        for (i = 0; i < a.m.d_model; i++) {
            double d = fabs((double)ob[i] - (double)oa[i]) / fmax(1.0, fabs((double)oa[i]));
            if (!(d <= worst)) worst = d;   /* NaN counts as the worst */
        }
        free(x); free(oa); free(ob);
    }
    {
        uint32_t n = tokens < window ? tokens : window;
        int8_t  *kc = (int8_t *)calloc((size_t)n * a.m.k_dim, 1);
        int8_t  *vc = (int8_t *)calloc((size_t)n * a.m.v_dim, 1);
        float   *ks = (float *)calloc((size_t)n * a.m.n_kv_heads, sizeof(float));
        float   *vs = (float *)calloc((size_t)n * a.m.n_kv_heads, sizeof(float));
        if (read_cache(h, 0, 0, 0, n, kc, vc, ks, vs) != 0) { fprintf(stderr, "read_cache\n"); return 3; }
        if (memcmp(kc, a.m.k_cache, (size_t)n * a.m.k_dim)) bad |= 1;
        if (memcmp(vc, a.m.v_cache, (size_t)n * a.m.v_dim)) bad |= 2;
        if (memcmp(ks, a.m.k_scale, (size_t)n * a.m.n_kv_heads * sizeof(float))) bad |= 4;
        if (memcmp(vs, a.m.v_scale, (size_t)n * a.m.n_kv_heads * sizeof(float))) bad |= 8;
        /* The hooked engine's own C caches stay untouched: the library owns the KV. */
        for (i = 0; i < (uint32_t)(n * a.m.k_dim); i++) if (b.m.k_cache[i]) { bad |= 16; break; }
        free(kc); free(vc); free(ks); free(vs);
    }
    if (!(worst <= 1e-3)) bad |= 32;
    g_ops->close(h);
    printf("hook_session tokens %u window %u n_sink %u worst_rel %.3e kv_mismatch_bits %d %s\n", tokens, window,
           n_sink, worst, bad, bad ? "FAIL" : "PASS");
    return bad ? 1 : 0;
}
