/*
 * iq_oracle_model.c -- CPU restatement of the reference's quantized model
 * forward pass, one row at a time.
 *
 * TEST INFRASTRUCTURE ONLY (see iq_oracle.h).  Built with -ffp-contract=off.
 *
 * Follows, file by file (paths in the ybrs/inferq tree):
 *   src/qwen/quantized_model.rs:654-752   forward_inner (embed, layers, final norm, LM head)
 *   src/qwen/quantized_layer.rs:101-236   layer wrappers, gguf_rms_norm
 *   src/qwen/quantized_deltanet.rs:517-759 DeltaNet mixer (conv, L2 norm, beta/alpha, gated norm)
 *   src/qwen/deltanet.rs:122-217          recurrent delta rule
 *   src/qwen/quantized_attention.rs:155-178, 409-589, 833-851  gated attention
 *   src/qwen/moe.rs:21-54                 softmax top-k routing
 *   src/qwen/quantized_moe.rs:237-460     routed + shared experts, ordered accumulation
 *   src/qwen/quantized_mtp.rs:175-227     MTP predictor block
 * Every projection goes through or_qmatvec in the reference lane order.
 * A multi-row pass of the reference equals its rows run one at a time
 * (per-row matmuls, serial recurrence, causal attention), so the oracle
 * evaluates passes of up to 8 rows, one row per step inside each (order 2:
 * the wide pass's 512-row chunks).
 */
#include "iq_oracle.h"
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct or_config {
    int32_t hidden_size, num_hidden_layers, vocab_size;
    int32_t num_attention_heads, num_key_value_heads, head_dim, rotary_dim;
    int32_t linear_num_key_heads, linear_num_value_heads, linear_key_head_dim, linear_value_head_dim;
    int32_t linear_conv_kernel_dim;
    int32_t num_experts, num_experts_per_tok, moe_intermediate_size, shared_expert_intermediate_size;
    int32_t full_attention_interval, mtp_num_hidden_layers, norm_topk_prob, value_heads_tiled;
    int32_t max_position_embeddings;
    float rms_norm_eps;
    double rope_theta;
} or_config;

typedef struct or_tensor {
    const char* name;
    int32_t dtype;
    int32_t ndim;
    int64_t shape[4];
    const void* data;
    int32_t location;
} or_tensor;

typedef struct { int dt; int64_t rows, cols; const uint8_t* p; } mat_t;

typedef struct {
    int full;
    const float *attn_norm, *post_norm;
    /* DeltaNet */
    mat_t qkv, z, ba, beta, alpha, out;
    int ba_fused;
    const float *conv_w, *ssm_a, *dt_bias, *ssm_norm;
    /* attention */
    mat_t q, k, v, o;
    const float *q_norm, *k_norm;
    /* MoE */
    mat_t router, gate, up, down, sh_gate, sh_up, sh_down;
    const float* selector;
} layer_t;

typedef struct or_model {
    or_config c;
    mat_t embed, lm_head;
    const float* out_norm;
    layer_t* layers;
    int has_mtp;
    layer_t mtp;
    const float *enorm, *hnorm, *head_norm;
    mat_t eh_proj;
} or_model;

typedef struct {
    float* conv;  /* [conv_dim][K-1] */
    float* rec;   /* [nv][dk][dv] */
    float* keys;  /* [max_pos][nkv][hd] */
    float* values;
    float** snap_conv;  /* snapshots after each row of a pass (or NULL) */
    float** snap_rec;
} lstate_t;

typedef struct or_state {
    int64_t position, max_pos;
    int nlayers;
    lstate_t* l;
    lstate_t mtp;
    int64_t mtp_position;
    /* verification snapshots (QuantizedStateSnapshots, quantized_model.rs:99-204):
     * with snap_rows > 0, a pass stores each DeltaNet layer's conv and
     * recurrent state after its rows 0..snap_rows-2, so a rollback is a copy */
    int snap_rows;
    int64_t snap_pos0;  /* position of the last pass's row 0 */
    int snap_taken;     /* rows of the last pass */
} or_state;

/* --------------------------------------------------------------- helpers */
static const or_tensor* find(const or_tensor* t, int n, const char* name) {
    for (int i = 0; i < n; i++)
        if (!strcmp(t[i].name, name)) return &t[i];
    return NULL;
}
static int getmat(const or_tensor* t, int n, const char* name, mat_t* m) {
    const or_tensor* x = find(t, n, name);
    if (!x) return -1;
    m->dt = x->dtype;
    m->cols = x->shape[x->ndim - 1];
    m->rows = 1;
    for (int i = 0; i < x->ndim - 1; i++) m->rows *= x->shape[i];
    m->p = (const uint8_t*)x->data;
    return 0;
}
static const float* getvec(const or_tensor* t, int n, const char* name) {
    const or_tensor* x = find(t, n, name);
    return x ? (const float*)x->data : NULL;
}

/* Accumulation orders: 0 = the reference's (AVX2 lane order of every
 * projection, sequential sums; the default), 1 = the device's 8-row passes
 * (block-chunk GEMV order, the device's RMSNorm sum), 2 = the device's wide
 * prefill pass (dense blocks in one chunk, experts split as on the device,
 * the device's RMSNorm sum, and passes of up to 512 rows whose DeltaNet rows
 * before the final block of 8 run in the chunked form, delta_chunk).  1 and 2
 * isolate f32-order effects from everything else in the parity tests. */
static int g_order = 0;
void or_set_gemv_order(int order) { g_order = order; }

/* The device's chunk count for a matrix shape (a function of shape only). */
static int device_ksplit(int dt, int64_t rows, int64_t cols, int expert) {
    if (dt == OR_F32) return 1;
    int units = (int)(dt == OR_Q8_0 ? cols / 128 : cols / 256);
    int64_t target = expert ? 32 : 148 * 32;
    int ks = 1;
    while (ks < 8 && units % (ks * 2) == 0 && (rows / 16) * ks < target) ks *= 2;
    return ks;
}

/* y[rows] = W x  (one input row) */
/* The chunk count of the device order for a matrix: `expert` 0 dense, 1 a
 * routed expert, 2 the shared expert.  Order 2 is the wide prefill pass's:
 * dense and shared matrices in one chunk (the tensor-core products), routed
 * experts as the GEMV splits them. */
static int order_ksplit(int dt, int64_t n, int64_t cols, int expert) {
    if (g_order == 2) return expert == 1 ? device_ksplit(dt, n, cols, 1) : 1;
    return g_order ? device_ksplit(dt, n, cols, expert != 0) : 1;
}
static void matvec_n(const mat_t* m, const uint8_t* p, int64_t n, const float* x, float* y, int expert) {
    or_qmatvec(m->dt, p, n, m->cols, x, 1, y, g_order ? 1 : 0, order_ksplit(m->dt, n, m->cols, expert));
}
static void matvec(const mat_t* m, const float* x, float* y) { matvec_n(m, m->p, m->rows, x, y, 0); }
/* R input rows x [R][cols] -> y [R][n] (each weight row read once for all R,
 * the reference's multi-row pass; every output is computed exactly as for a
 * single row) */
static void matvec_nk(const mat_t* m, const uint8_t* p, int64_t n, const float* x, int R, float* y, int expert) {
    or_qmatvec(m->dt, p, n, m->cols, x, R, y, g_order ? 1 : 0, order_ksplit(m->dt, n, m->cols, expert));
}
static void matvec_k(const mat_t* m, const float* x, int R, float* y) { matvec_nk(m, m->p, m->rows, x, R, y, 0); }
/* an expert-class matrix (routed or shared expert) */
static void matvec_e(const mat_t* m, const float* x, float* y) { matvec_n(m, m->p, m->rows, x, y, 1); }
/* rows [r0, r0+n) of a stacked expert matrix */
static void matvec_rows(const mat_t* m, int64_t r0, int64_t n, const float* x, float* y) {
    matvec_n(m, m->p + r0 * or_row_bytes(m->dt, m->cols), n, x, y, 1);
}

static float sigmoid_ref(float v) { return 1.f / (1.f + expf(-v)); }
static float softplus_ref(float v) { return v > 20.f ? v : v < -20.f ? expf(v) : log1pf(expf(v)); }

/* Rounding-level perturbation (a diagnostic of the reference arithmetic's
 * own conditioning, off by default): mode 1 moves every RMSNorm output
 * element by one ulp (odd elements up, even ones down), mode 2 the other
 * way, as a different but equally valid summation order would move them. */
static int g_perturb = 0;
void or_set_perturb(int on) { g_perturb = on; }

/* gguf_rms_norm (quantized_layer.rs:230-236): x / sqrt(mean(x^2) + eps) * w */
/* The device row-prep kernel's sum of squares (inferq_b200/csrc/layout.cu
 * prep_rows_kernel), used by the device orders: thread (warp w, lane l) of
 * 256 takes the 256-element blocks b = w + 8j and in each the elements
 * 32 (l & 7) + 16 (i / 4) + 4 (l >> 3) + (i % 4), i = 0..7, as fused
 * multiply-adds; each warp's lanes combine by the xor butterfly 16, 8, 4, 2,
 * 1; the eight warp sums are added in warp order. */
static float dev_sum_squares(const float* x, int n) {
    const int nb = (n + 255) / 256;
    float red[8];
    for (int wp = 0; wp < 8; wp++) {
        float lanes[32], nx[32];
        for (int l = 0; l < 32; l++) {
            float acc = 0.f;
            for (int b = wp; b < nb; b += 8)
                for (int i = 0; i < 8; i++) {
                    int idx = b * 256 + 32 * (l & 7) + 16 * (i / 4) + 4 * (l >> 3) + (i % 4);
                    float v = idx < n ? x[idx] : 0.f;
                    acc = fmaf(v, v, acc);
                }
            lanes[l] = acc;
        }
        for (int m = 16; m >= 1; m >>= 1) {
            for (int l = 0; l < 32; l++) nx[l] = lanes[l] + lanes[l ^ m];
            memcpy(lanes, nx, sizeof lanes);
        }
        red[wp] = lanes[0];
    }
    float t = red[0];
    for (int i = 1; i < 8; i++) t = t + red[i];
    return t;
}

static void rms_norm(const float* x, const float* w, int n, float eps, float* out) {
    float ss = 0.f;
    if (g_order) ss = dev_sum_squares(x, n);
    else
        for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float var = ss * (float)(1.0 / (double)n);
    float den = sqrtf(var + eps);
    for (int i = 0; i < n; i++) out[i] = (x[i] / den) * w[i];
    if (g_perturb)
        for (int i = 0; i < n; i++)
            out[i] = nextafterf(out[i], ((i & 1) ^ (g_perturb == 2)) ? INFINITY : -INFINITY);
}

void or_rms_norm(const float* x, const float* w, int n, float eps, float* out) { rms_norm(x, w, n, eps, out); }

/* accepted_draft_prefix (runtime.rs:2225-2236): the number of leading
 * drafts equal to the greedy argmax of the row before them; logits holds
 * ndrafts+1 rows of `vocab`. */
int or_accepted_prefix(const uint32_t* drafts, int ndrafts, const float* logits, int64_t vocab) {
    int a = 0;
    while (a < ndrafts && or_argmax(logits + (int64_t)a * vocab, vocab) == (int64_t)drafts[a]) a++;
    return a;
}

/* ------------------------------------------------------------- creation */
#define REQ(x) do { if (!(x)) { free(m->layers); free(m); return NULL; } } while (0)

static int load_moe(const or_tensor* t, int n, const char* p, layer_t* L) {
    char b[256];
    snprintf(b, sizeof b, "%s.ffn_gate_inp.weight", p); if (getmat(t, n, b, &L->router)) return -1;
    snprintf(b, sizeof b, "%s.ffn_gate_exps.weight", p); if (getmat(t, n, b, &L->gate)) return -1;
    snprintf(b, sizeof b, "%s.ffn_up_exps.weight", p); if (getmat(t, n, b, &L->up)) return -1;
    snprintf(b, sizeof b, "%s.ffn_down_exps.weight", p); if (getmat(t, n, b, &L->down)) return -1;
    snprintf(b, sizeof b, "%s.ffn_gate_shexp.weight", p); if (getmat(t, n, b, &L->sh_gate)) return -1;
    snprintf(b, sizeof b, "%s.ffn_up_shexp.weight", p); if (getmat(t, n, b, &L->sh_up)) return -1;
    snprintf(b, sizeof b, "%s.ffn_down_shexp.weight", p); if (getmat(t, n, b, &L->sh_down)) return -1;
    snprintf(b, sizeof b, "%s.ffn_gate_inp_shexp.weight", p); if (!(L->selector = getvec(t, n, b))) return -1;
    return 0;
}
static int load_attn(const or_tensor* t, int n, const char* p, layer_t* L) {
    char b[256];
    L->full = 1;
    snprintf(b, sizeof b, "%s.attn_q.weight", p); if (getmat(t, n, b, &L->q)) return -1;
    snprintf(b, sizeof b, "%s.attn_k.weight", p); if (getmat(t, n, b, &L->k)) return -1;
    snprintf(b, sizeof b, "%s.attn_v.weight", p); if (getmat(t, n, b, &L->v)) return -1;
    snprintf(b, sizeof b, "%s.attn_output.weight", p); if (getmat(t, n, b, &L->o)) return -1;
    snprintf(b, sizeof b, "%s.attn_q_norm.weight", p); if (!(L->q_norm = getvec(t, n, b))) return -1;
    snprintf(b, sizeof b, "%s.attn_k_norm.weight", p); if (!(L->k_norm = getvec(t, n, b))) return -1;
    return 0;
}
static int load_norms(const or_tensor* t, int n, const char* p, layer_t* L) {
    char b[256];
    snprintf(b, sizeof b, "%s.attn_norm.weight", p); if (!(L->attn_norm = getvec(t, n, b))) return -1;
    snprintf(b, sizeof b, "%s.post_attention_norm.weight", p); if (!(L->post_norm = getvec(t, n, b))) return -1;
    return 0;
}

or_model* or_model_create(const or_config* c, const or_tensor* t, int n) {
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    m->c = *c;
    m->layers = (layer_t*)calloc((size_t)c->num_hidden_layers, sizeof(layer_t));
    REQ(!getmat(t, n, "token_embd.weight", &m->embed));
    REQ(!getmat(t, n, "output.weight", &m->lm_head));
    REQ(m->out_norm = getvec(t, n, "output_norm.weight"));
    char p[64], b[256];
    for (int l = 0; l < c->num_hidden_layers; l++) {
        layer_t* L = &m->layers[l];
        snprintf(p, sizeof p, "blk.%d", l);
        REQ(!load_norms(t, n, p, L));
        if ((l + 1) % c->full_attention_interval == 0) {
            REQ(!load_attn(t, n, p, L));
        } else {
            snprintf(b, sizeof b, "%s.attn_qkv.weight", p); REQ(!getmat(t, n, b, &L->qkv));
            snprintf(b, sizeof b, "%s.attn_gate.weight", p); REQ(!getmat(t, n, b, &L->z));
            snprintf(b, sizeof b, "%s.ssm_ba.weight", p);
            if (!getmat(t, n, b, &L->ba)) L->ba_fused = 1;
            else {
                snprintf(b, sizeof b, "%s.ssm_beta.weight", p); REQ(!getmat(t, n, b, &L->beta));
                snprintf(b, sizeof b, "%s.ssm_alpha.weight", p); REQ(!getmat(t, n, b, &L->alpha));
            }
            snprintf(b, sizeof b, "%s.ssm_out.weight", p); REQ(!getmat(t, n, b, &L->out));
            snprintf(b, sizeof b, "%s.ssm_conv1d.weight", p); REQ(L->conv_w = getvec(t, n, b));
            snprintf(b, sizeof b, "%s.ssm_a", p); REQ(L->ssm_a = getvec(t, n, b));
            snprintf(b, sizeof b, "%s.ssm_dt.bias", p); REQ(L->dt_bias = getvec(t, n, b));
            snprintf(b, sizeof b, "%s.ssm_norm.weight", p); REQ(L->ssm_norm = getvec(t, n, b));
        }
        REQ(!load_moe(t, n, p, L));
    }
    if (c->mtp_num_hidden_layers == 1) {
        m->has_mtp = 1;
        snprintf(p, sizeof p, "blk.%d", c->num_hidden_layers);
        REQ(!load_norms(t, n, p, &m->mtp));
        REQ(!load_attn(t, n, p, &m->mtp));
        REQ(!load_moe(t, n, p, &m->mtp));
        snprintf(b, sizeof b, "%s.nextn.enorm.weight", p); REQ(m->enorm = getvec(t, n, b));
        snprintf(b, sizeof b, "%s.nextn.hnorm.weight", p); REQ(m->hnorm = getvec(t, n, b));
        snprintf(b, sizeof b, "%s.nextn.shared_head_norm.weight", p); REQ(m->head_norm = getvec(t, n, b));
        snprintf(b, sizeof b, "%s.nextn.eh_proj.weight", p); REQ(!getmat(t, n, b, &m->eh_proj));
    }
    return m;
}

void or_model_destroy(or_model* m) {
    if (!m) return;
    free(m->layers);
    free(m);
}

static void lstate_alloc(const or_config* c, int full, int64_t max_pos, lstate_t* s) {
    memset(s, 0, sizeof *s);
    if (full) {
        size_t kv = (size_t)max_pos * c->num_key_value_heads * c->head_dim;
        s->keys = (float*)calloc(kv, 4);
        s->values = (float*)calloc(kv, 4);
    } else {
        int64_t conv_dim = 2 * (int64_t)c->linear_num_key_heads * c->linear_key_head_dim +
                           (int64_t)c->linear_num_value_heads * c->linear_value_head_dim;
        s->conv = (float*)calloc((size_t)(conv_dim * (c->linear_conv_kernel_dim - 1) + 1), 4);
        s->rec = (float*)calloc((size_t)c->linear_num_value_heads * c->linear_key_head_dim * c->linear_value_head_dim, 4);
    }
}
static void lstate_free(lstate_t* s) { free(s->conv); free(s->rec); free(s->keys); free(s->values); }

or_state* or_state_create(const or_model* m, int64_t max_pos) {
    or_state* s = (or_state*)calloc(1, sizeof(or_state));
    s->max_pos = max_pos;
    s->nlayers = m->c.num_hidden_layers;
    s->l = (lstate_t*)calloc((size_t)s->nlayers, sizeof(lstate_t));
    for (int i = 0; i < s->nlayers; i++) lstate_alloc(&m->c, m->layers[i].full, max_pos, &s->l[i]);
    if (m->has_mtp) lstate_alloc(&m->c, 1, max_pos, &s->mtp);
    return s;
}

/* Keep snapshots for passes of up to `rows` rows (0 turns them off). */
int or_state_enable_snapshots(const or_model* m, or_state* s, int rows) {
    const or_config* c = &m->c;
    int64_t conv_n = (2 * (int64_t)c->linear_num_key_heads * c->linear_key_head_dim +
                      (int64_t)c->linear_num_value_heads * c->linear_value_head_dim) * (c->linear_conv_kernel_dim - 1);
    int64_t rec_n = (int64_t)c->linear_num_value_heads * c->linear_key_head_dim * c->linear_value_head_dim;
    if (rows > 8 || rows < 0 || s->snap_rows) return -1;
    s->snap_rows = rows;
    for (int i = 0; i < s->nlayers; i++) {
        if (m->layers[i].full || rows < 2) continue;
        lstate_t* L = &s->l[i];
        L->snap_conv = (float**)calloc((size_t)rows, sizeof(float*));
        L->snap_rec = (float**)calloc((size_t)rows, sizeof(float*));
        for (int r = 0; r + 1 < rows; r++) {
            L->snap_conv[r] = (float*)malloc((size_t)(conv_n + 1) * 4);
            L->snap_rec[r] = (float*)malloc((size_t)rec_n * 4);
        }
    }
    return 0;
}

/* Keep the first `committed` rows of the last pass (rollback,
 * quantized_model.rs:177-204): DeltaNet state from the snapshot after row
 * committed-1, KV cache truncated by the position. */
int or_state_rollback(const or_model* m, or_state* s, int committed) {
    const or_config* c = &m->c;
    if (committed < 1 || committed > s->snap_taken) return -1;
    if (committed == s->snap_taken) return 0;
    if (!s->snap_rows) return -2;
    int64_t conv_n = (2 * (int64_t)c->linear_num_key_heads * c->linear_key_head_dim +
                      (int64_t)c->linear_num_value_heads * c->linear_value_head_dim) * (c->linear_conv_kernel_dim - 1);
    int64_t rec_n = (int64_t)c->linear_num_value_heads * c->linear_key_head_dim * c->linear_value_head_dim;
    for (int i = 0; i < s->nlayers; i++) {
        if (m->layers[i].full) continue;
        lstate_t* L = &s->l[i];
        memcpy(L->conv, L->snap_conv[committed - 1], (size_t)conv_n * 4);
        memcpy(L->rec, L->snap_rec[committed - 1], (size_t)rec_n * 4);
    }
    s->position = s->snap_pos0 + committed;
    s->snap_taken = committed;
    return 0;
}

void or_state_destroy(or_state* s) {
    if (!s) return;
    for (int i = 0; i < s->nlayers; i++) {
        lstate_t* L = &s->l[i];
        if (L->snap_conv) {
            for (int r = 0; r + 1 < s->snap_rows; r++) { free(L->snap_conv[r]); free(L->snap_rec[r]); }
            free(L->snap_conv); free(L->snap_rec);
        }
    }
    for (int i = 0; i < s->nlayers; i++) lstate_free(&s->l[i]);
    lstate_free(&s->mtp);
    free(s->l);
    free(s);
}

/* Deep copy (the snapshot a rollback restores). */
void or_state_copy(const or_model* m, or_state* dst, const or_state* src) {
    const or_config* c = &m->c;
    int64_t conv_dim = 2 * (int64_t)c->linear_num_key_heads * c->linear_key_head_dim +
                       (int64_t)c->linear_num_value_heads * c->linear_value_head_dim;
    size_t kv = (size_t)src->max_pos * c->num_key_value_heads * c->head_dim;
    size_t rec = (size_t)c->linear_num_value_heads * c->linear_key_head_dim * c->linear_value_head_dim;
    for (int i = 0; i < src->nlayers; i++) {
        if (m->layers[i].full) {
            memcpy(dst->l[i].keys, src->l[i].keys, kv * 4);
            memcpy(dst->l[i].values, src->l[i].values, kv * 4);
        } else {
            memcpy(dst->l[i].conv, src->l[i].conv, (size_t)(conv_dim * (c->linear_conv_kernel_dim - 1) + 1) * 4);
            memcpy(dst->l[i].rec, src->l[i].rec, rec * 4);
        }
    }
    if (m->has_mtp) {
        memcpy(dst->mtp.keys, src->mtp.keys, kv * 4);
        memcpy(dst->mtp.values, src->mtp.values, kv * 4);
    }
    dst->position = src->position;
    dst->mtp_position = src->mtp_position;
}

int64_t or_state_position(const or_state* s) { return s->position; }

/* ------------------------------------------------------------ DeltaNet */
/* causal_depthwise_conv_step + SiLU (quantized_deltanet.rs:733-759): per
 * channel, sum = w[K-1]*x + sum_tap w[tap]*history[tap] (each product
 * rounded, added in tap order), output silu(sum), history shifted left and
 * the input appended.  state is [channels][K-1]. */
void or_conv_step(const float* input, const float* weights, int channels, int kernel, float* state, float* output) {
    for (int ch = 0; ch < channels; ch++) {
        const float* w = weights + (int64_t)ch * kernel;
        float* hist = state + (int64_t)ch * (kernel - 1);
        float sum = w[kernel - 1] * input[ch];
        for (int tap = 0; tap < kernel - 1; tap++) sum += w[tap] * hist[tap];
        output[ch] = sum * sigmoid_ref(sum);
        for (int tap = 0; tap + 1 < kernel - 1; tap++) hist[tap] = hist[tap + 1];
        if (kernel > 1) hist[kernel - 2] = input[ch];
    }
}

/* normalize (quantized_deltanet.rs:724-731): x * (sum x^2 + 1e-6)^-1/2, the
 * sum in element order. */
void or_l2_normalize(float* a, int n) {
    float ss = 0.f;
    for (int i = 0; i < n; i++) ss += a[i] * a[i];
    float scale = 1.f / sqrtf(ss + 1e-6f);
    for (int i = 0; i < n; i++) a[i] *= scale;
}

float or_softplus(float v) { return softplus_ref(v); }

/* ValueHeadLayout::index (quantized_deltanet.rs:358-376): the value head of
 * (key head, repeat): GroupedByKeyHead key*ratio + repeat (Qwen3-Next),
 * TiledByRepeat repeat*key_heads + key (Qwen3.6). */
int or_value_head(int key, int repeat, int key_heads, int ratio, int tiled) {
    return tiled ? repeat * key_heads + key : key * ratio + repeat;
}

/* delta_head_step (deltanet.rs:170-217) on one head's [dk][dv] state:
 * S *= exp(g); pred_j = sum_i S[i][j] k[i]; delta_j = (v_j - pred_j) beta;
 * S[i][j] += k[i] delta_j; out_j = sum_i S[i][j] q[i] q_scale, every sum in
 * key-row order and every product rounded. */
static void delta_head_step(const float* qq, const float* kk, const float* vv, float g, float beta, int dk, int dv,
                            float q_scale, float* S, float* out_h) {
    float decay = expf(g);
    for (int i = 0; i < dk * dv; i++) S[i] *= decay;
    for (int j = 0; j < dv; j++) out_h[j] = 0.f;
    for (int i = 0; i < dk; i++) for (int j = 0; j < dv; j++) out_h[j] += S[i * dv + j] * kk[i];
    for (int j = 0; j < dv; j++) out_h[j] = (vv[j] - out_h[j]) * beta;
    for (int i = 0; i < dk; i++) for (int j = 0; j < dv; j++) S[i * dv + j] += kk[i] * out_h[j];
    for (int j = 0; j < dv; j++) out_h[j] = 0.f;
    for (int i = 0; i < dk; i++) for (int j = 0; j < dv; j++) out_h[j] += S[i * dv + j] * qq[i] * q_scale;
}

/* recurrent_delta_step (deltanet.rs:122-166): every head on its own state
 * block [heads][dk][dv]; q_scale = 1/sqrt(dk). */
void or_delta_step(const float* q, const float* k, const float* v, const float* g, const float* beta, int heads,
                   int dk, int dv, float* state, float* out) {
    float q_scale = 1.f / sqrtf((float)dk);
    for (int h = 0; h < heads; h++)
        delta_head_step(q + h * dk, k + h * dk, v + h * dv, g[h], beta[h], dk, dv, q_scale,
                        state + (int64_t)h * dk * dv, out + h * dv);
}

/* ------------------------------------------------ chunked recurrence */
/* The device's chunked form of the recurrence for the rows of a wide pass
 * before its final block (order 2; inferq_b200/csrc/deltanet_chunk.cu
 * states the algebra).  Same arithmetic as delta_head_step up to f32
 * rounding order; this restates the device's order exactly: key-dimension
 * dots sequential; U and W of delta = U - W S0 by forward substitution in s
 * order; W_t S0 and S0^T q in eight parts (part p: rows p dk/8 .. (p+1) dk/8 - 1)
 * combined as
 * ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)), sums over s split s = p (mod 8) and
 * combined the same way, decays as exp of cumulative log-decay differences. */
static float expd(float x) { return (float)exp((double)x); }
static float tree8(const float* p) {
    return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
}
#define CHUNK 32
/* One value head over C rows: q/k [C][ld_qk], v [C][ld_v], beta/lg [C];
 * S [dk][dv] advanced in place; o [C][ld_o] raw outputs. */
static void delta_chunk(const float* q, const float* k, int ld_qk, const float* v, int ld_v, const float* beta,
                        const float* lg, int C, int dk, int dv, float* S, float* o, int ld_o) {
    static float A[CHUNK][CHUNK], M[CHUNK][CHUNK], D[CHUNK][128], Lc[CHUNK], E[CHUNK], W[CHUNK];
    const int kp = dk / 8;
    const float qscale = 1.f / sqrtf((float)dk);
    float l = 0.f;
    for (int t = 0; t < C; t++) { l = l + lg[t]; Lc[t] = l; E[t] = expd(l); }
    for (int s = 0; s < C; s++) W[s] = expd(Lc[C - 1] - Lc[s]);
    for (int t = 0; t < C; t++)
        for (int s = 0; s < C; s++) {
            float m = 0.f, aa = 0.f;
            if (s <= t) {
                float r = expd(Lc[t] - Lc[s]);
                float qk = 0.f;
                for (int i = 0; i < dk; i++) qk = qk + q[t * ld_qk + i] * k[s * ld_qk + i];
                m = r * qk;
                if (s < t) {
                    float kk = 0.f;
                    for (int i = 0; i < dk; i++) kk = kk + k[t * ld_qk + i] * k[s * ld_qk + i];
                    aa = (beta[t] * r) * kk;
                }
            }
            M[t][s] = m;
            A[t][s] = aa;
        }
    /* U_t = beta_t v_t - sum_{s<t} A U_s, W_t = (beta_t e_t) k_t - sum_{s<t} A W_s */
    static float U[CHUNK][128], Wk[CHUNK][128];
    for (int j = 0; j < dv; j++)
        for (int t = 0; t < C; t++) {
            float acc = 0.f;
            for (int s = 0; s < t; s++) acc = acc + A[t][s] * U[s][j];
            U[t][j] = beta[t] * v[t * ld_v + j] - acc;
        }
    for (int i = 0; i < dk; i++)
        for (int t = 0; t < C; t++) {
            float acc = 0.f;
            for (int s = 0; s < t; s++) acc = acc + A[t][s] * Wk[s][i];
            Wk[t][i] = (beta[t] * E[t]) * k[t * ld_qk + i] - acc;
        }
    for (int j = 0; j < dv; j++) {
        float R[CHUNK];
        for (int t = 0; t < C; t++) {
            float pw[8], pq[8];
            for (int p = 0; p < 8; p++) {
                float a1 = 0.f, a2 = 0.f;
                for (int ii = 0; ii < kp; ii++) {
                    int i = p * kp + ii;
                    a1 = a1 + S[i * dv + j] * Wk[t][i];
                    a2 = a2 + S[i * dv + j] * q[t * ld_qk + i];
                }
                pw[p] = a1; pq[p] = a2;
            }
            D[t][j] = U[t][j] - tree8(pw);
            R[t] = tree8(pq);
        }
        for (int t = 0; t < C; t++) {
            float po[8];
            for (int p = 0; p < 8; p++) {
                float acc = 0.f;
                for (int s = p; s <= t; s += 8) acc = acc + M[t][s] * D[s][j];
                po[p] = acc;
            }
            o[t * ld_o + j] = qscale * (E[t] * R[t] + tree8(po));
        }
        for (int i = 0; i < dk; i++) {
            float acc = E[C - 1] * S[i * dv + j];
            for (int s = 0; s < C; s++) acc = acc + (W[s] * k[s * ld_qk + i]) * D[s][j];
            S[i * dv + j] = acc;
        }
    }
}
/* The chunked form over C <= 32 rows of one value head, exported for the
 * tests that compare it with the sequential rule: q, k [C][dk] (normalized),
 * v [C][dv], beta and log-decay [C]; S [dk][dv] advanced in place; o [C][dv]. */
int or_delta_chunk(const float* q, const float* k, const float* v, const float* beta, const float* lg, int C, int dk,
                   int dv, float* S, float* o) {
    if (C < 1 || C > CHUNK || dk % 8 || dv > 128 || dv < 1) return -1;
    delta_chunk(q, k, dk, v, dv, beta, lg, C, dk, dv, S, o, dv);
    return 0;
}

static int chunk_supported(const or_config* c) {
    int nk = c->linear_num_key_heads, nv = c->linear_num_value_heads, dk = c->linear_key_head_dim;
    int dv = c->linear_value_head_dim, K = c->linear_conv_kernel_dim;
    return (dk == 64 || dk == 128) && dv % 16 == 0 && dv >= 16 && dv <= 128 && nv <= 128 && 2 * nk <= 64 &&
           K >= 2 && K <= 4 && (2 * nk * dk + nv * dv) * 4 <= 200 * 1024;
}

/* The DeltaNet mixer over R rows x [R][H] -> out [R][H]
 * (quantized_deltanet.rs:517-703): projections of all rows, then per row in
 * order the conv step, L2 norms, beta/decay and the delta rule, then the
 * gated norm and the output projection of all rows. */
static void delta_rows(const or_model* m, const layer_t* L, lstate_t* st, const float* x, int R, float* out) {
    const or_config* c = &m->c;
    const int nk = c->linear_num_key_heads, nv = c->linear_num_value_heads;
    const int dk = c->linear_key_head_dim, dv = c->linear_value_head_dim, K = c->linear_conv_kernel_dim;
    const int kd = nk * dk, vd = nv * dv, conv_dim = 2 * kd + vd, ratio = nv / nk;
    float* proj = (float*)malloc((size_t)R * conv_dim * 4);
    float* z = (float*)malloc((size_t)R * vd * 4);
    float* ba = (float*)malloc((size_t)R * 2 * nv * 4);
    float* tmp = (float*)malloc((size_t)R * nv * 4);
    float* cv = (float*)malloc((size_t)conv_dim * 4);
    float* g = (float*)malloc((size_t)R * vd * 4);
    matvec_k(&L->qkv, x, R, proj);
    matvec_k(&L->z, x, R, z);
    if (L->ba_fused) matvec_k(&L->ba, x, R, ba);
    else {
        matvec_k(&L->beta, x, R, tmp);
        for (int r = 0; r < R; r++) memcpy(ba + (int64_t)r * 2 * nv, tmp + (int64_t)r * nv, (size_t)nv * 4);
        matvec_k(&L->alpha, x, R, tmp);
        for (int r = 0; r < R; r++) memcpy(ba + (int64_t)r * 2 * nv + nv, tmp + (int64_t)r * nv, (size_t)nv * 4);
    }
    /* order 2 over a wide pass: the rows before the final block of up to 8 in
     * the chunked form (delta_chunk), the final block row by row */
    const int pre = (g_order == 2 && R > 8 && chunk_supported(c)) ? R - ((R - 1) % 8 + 1) : 0;
    float* oall = (float*)malloc((size_t)R * vd * 4);
    /* per row in order: conv step, L2 norms, beta and log-decay; each value
     * head's inputs collected (q/k repeated per value head) */
    float* cq = (float*)malloc((size_t)R * nv * dk * 4);
    float* ck = (float*)malloc((size_t)R * nv * dk * 4);
    float* cvv = (float*)malloc((size_t)R * vd * 4);
    float* cb = (float*)malloc((size_t)R * nv * 4);
    float* cl = (float*)malloc((size_t)R * nv * 4);
    for (int r = 0; r < R; r++) {
        const float* bar = ba + (int64_t)r * 2 * nv;
        or_conv_step(proj + (int64_t)r * conv_dim, L->conv_w, conv_dim, K, st->conv, cv);
        float* q = cv; float* k = cv + kd; const float* v = cv + 2 * kd;
        for (int kh = 0; kh < nk; kh++) {
            or_l2_normalize(q + kh * dk, dk);
            or_l2_normalize(k + kh * dk, dk);
        }
        for (int kh = 0; kh < nk; kh++)
            for (int rep = 0; rep < ratio; rep++) {
                int vh = or_value_head(kh, rep, nk, ratio, c->value_heads_tiled);
                float b, al;
                if (L->ba_fused) { int base = kh * 2 * ratio; b = bar[base + rep]; al = bar[base + ratio + rep]; }
                else { b = bar[vh]; al = bar[nv + vh]; }
                memcpy(cq + ((int64_t)r * nv + vh) * dk, q + kh * dk, (size_t)dk * 4);
                memcpy(ck + ((int64_t)r * nv + vh) * dk, k + kh * dk, (size_t)dk * 4);
                memcpy(cvv + (int64_t)r * vd + vh * dv, v + vh * dv, (size_t)dv * 4);
                cb[r * nv + vh] = sigmoid_ref(b);
                cl[r * nv + vh] = L->ssm_a[vh] * softplus_ref(al + L->dt_bias[vh]);
            }
        if (st->snap_conv && r + 1 < R)  /* entry state of the next row */
            memcpy(st->snap_conv[r], st->conv, (size_t)conv_dim * (K - 1) * 4);
    }
    /* the prefix of a wide pass in the chunked form, head by head */
    for (int vh = 0; vh < nv && pre > 0; vh++) {
        float bh[CHUNK], lh[CHUNK];
        for (int c0 = 0; c0 < pre; c0 += CHUNK) {
            int C = pre - c0 < CHUNK ? pre - c0 : CHUNK;
            for (int t = 0; t < C; t++) { bh[t] = cb[(c0 + t) * nv + vh]; lh[t] = cl[(c0 + t) * nv + vh]; }
            delta_chunk(cq + (int64_t)c0 * nv * dk + vh * dk, ck + (int64_t)c0 * nv * dk + vh * dk, nv * dk,
                        cvv + (int64_t)c0 * vd + vh * dv, vd, bh, lh, C, dk, dv,
                        st->rec + (int64_t)vh * dk * dv, oall + (int64_t)c0 * vd + vh * dv, vd);
        }
    }
    /* the remaining rows with the delta rule; the heads are independent, so
     * they run in parallel, each walking its rows in order */
    const float q_scale = 1.f / sqrtf((float)dk);
#pragma omp parallel for schedule(static)
    for (int vh = 0; vh < nv; vh++) {
        float* S = st->rec + (int64_t)vh * dk * dv;
        for (int r = pre; r < R; r++) {
            delta_head_step(cq + ((int64_t)r * nv + vh) * dk, ck + ((int64_t)r * nv + vh) * dk,
                            cvv + (int64_t)r * vd + vh * dv, cl[r * nv + vh], cb[r * nv + vh], dk, dv, q_scale, S,
                            oall + (int64_t)r * vd + vh * dv);
            if (st->snap_rec && r + 1 < R)  /* this head's part of the next row's entry state */
                memcpy(st->snap_rec[r] + (int64_t)vh * dk * dv, S, (size_t)dk * dv * 4);
        }
    }
    for (int r = 0; r < R; r++) {
        /* rms_norm_gated (norm.rs:16-25) per value head */
        for (int vh = 0; vh < nv; vh++) {
            const float* oh = oall + (int64_t)r * vd + vh * dv;
            float ss = 0.f;
            for (int j = 0; j < dv; j++) ss += oh[j] * oh[j];
            float den = sqrtf(ss * (float)(1.0 / dv) + c->rms_norm_eps);
            for (int j = 0; j < dv; j++) {
                float zz = z[(int64_t)r * vd + vh * dv + j];
                float silu = zz / (1.f + expf(-zz));
                g[(int64_t)r * vd + vh * dv + j] = ((oh[j] / den) * L->ssm_norm[j]) * silu;
            }
        }
    }
    free(oall); free(cq); free(ck); free(cvv); free(cb); free(cl);
    matvec_k(&L->out, g, R, out);
    free(proj); free(z); free(ba); free(tmp); free(cv); free(g);
}

/* ----------------------------------------------------------- attention */
static float dot8(const float* a, const float* b, int n) {  /* quantized_attention.rs:155-178 */
    float lanes[8] = {0};
    int full = n / 8 * 8;
    for (int i = 0; i < full; i += 8)
        for (int l = 0; l < 8; l++) lanes[l] += a[i + l] * b[i + l];
    float total = 0.f;
    for (int i = full; i < n; i++) total += a[i] * b[i];
    for (int l = 0; l < 8; l++) total += lanes[l];
    return total;
}
static void converted_norm(float* v, const float* w, int n, float eps) {  /* :833-839 */
    float ss = 0.f;
    for (int i = 0; i < n; i++) ss += v[i] * v[i];
    float var = ss / (float)n;
    float scale = 1.f / sqrtf(var + eps);
    for (int i = 0; i < n; i++) v[i] = v[i] * scale * w[i];
}
static void apply_rope(float* v, int64_t pos, int rd, double theta) {  /* :841-851 */
    int half = rd / 2;
    float orig[512];
    memcpy(orig, v, (size_t)rd * 4);
    for (int i = 0; i < half; i++) {
        double freq = 1.0 / pow(theta, (double)(2 * i) / (double)rd);
        double ang = (double)pos * freq;
        float s = (float)sin(ang), cs = (float)cos(ang);
        v[i] = orig[i] * cs - orig[half + i] * s;
        v[half + i] = orig[half + i] * cs + orig[i] * s;
    }
}

/* The per-head scan of one query row (quantized_attention.rs:409-589):
 * scores dot8(q, key) * (1/sqrt(hd)) over `positions` cached rows, softmax
 * (max, exp, sum in position order, divide), probability-weighted value sum
 * in position order, output times sigmoid(gate).  Query head h reads KV head
 * h / (nh / nkv).  q and gate of head h at qg + h*q_ld and + gate_off;
 * keys/values [positions][nkv][hd]; res [nh][hd]. */
int or_have_avx2(void);
int or_scalar_forced(void);
float or_dot8_avx2(const float* a, const float* b, int n);
void or_attend_values_avx2(float* o, float* scores, float den, const float* v, int64_t positions, int64_t stride,
                           int hd);

static void attend_row(const float* qg, int q_ld, int gate_off, const float* keys, const float* values, int nh, int nkv,
                       int hd, int64_t positions, float* scores_all, float* res) {
    /* scores_all: nh rows of `positions` floats (one per head: the heads are
     * independent and run in parallel, each in its own order).  The AVX2
     * forms of the two inner loops give the same bits (iq_oracle_avx2.c). */
    const int G = nh / nkv;
    float scale = 1.f / sqrtf((float)hd);
    static int avx2 = -1;
    if (avx2 < 0) avx2 = or_have_avx2();
    const int vec = avx2 && !or_scalar_forced();
#pragma omp parallel for schedule(static)
    for (int h = 0; h < nh; h++) {
        float* scores = scores_all + (int64_t)h * positions;
        const float* q = qg + (int64_t)h * q_ld;
        const float* gate = q + gate_off;
        int kvh = h / G;
        float mx = -INFINITY;
        for (int64_t p = 0; p < positions; p++) {
            const float* kr = keys + (p * nkv + kvh) * hd;
            scores[p] = (vec ? or_dot8_avx2(q, kr, hd) : dot8(q, kr, hd)) * scale;
            if (scores[p] > mx) mx = scores[p];
        }
        float den = 0.f;
        for (int64_t p = 0; p < positions; p++) { scores[p] = expf(scores[p] - mx); den += scores[p]; }
        float* o = res + (int64_t)h * hd;
        for (int d = 0; d < hd; d++) o[d] = 0.f;
        if (vec) {
            or_attend_values_avx2(o, scores, den, values + (int64_t)kvh * hd, positions, (int64_t)nkv * hd, hd);
        } else {
            for (int64_t p = 0; p < positions; p++) {
                float prob = scores[p] / den;
                const float* vr = values + (p * nkv + kvh) * hd;
                for (int d = 0; d < hd; d++) o[d] += prob * vr[d];
            }
        }
        for (int d = 0; d < hd; d++) o[d] *= sigmoid_ref(gate[d]);
    }
}

/* Exported forms of the attention pieces for known-answer tests. */
float or_dot8(const float* a, const float* b, int n) { return dot8(a, b, n); }
void or_converted_norm(float* v, const float* w, int n, float eps) { converted_norm(v, w, n, eps); }
void or_attend(const float* q, const float* gate, const float* keys, const float* values, int nh, int nkv, int hd,
               int64_t positions, float* out) {
    /* q and gate as [nh][hd] each: interleave into the layer's [q | gate] rows */
    float* qg = (float*)malloc((size_t)nh * 2 * hd * 4);
    float* scores = (float*)malloc((size_t)nh * (positions > 0 ? positions : 1) * 4);
    for (int h = 0; h < nh; h++) {
        memcpy(qg + (int64_t)h * 2 * hd, q + (int64_t)h * hd, (size_t)hd * 4);
        memcpy(qg + (int64_t)h * 2 * hd + hd, gate + (int64_t)h * hd, (size_t)hd * 4);
    }
    attend_row(qg, 2 * hd, hd, keys, values, nh, nkv, hd, positions, scores, out);
    free(qg); free(scores);
}

/* Gated attention over R rows at positions pos .. pos+R-1
 * (quantized_attention.rs:409-507): projections of all rows, then per row in
 * order its K/V appended and its causal scan, then the output projection. */
static void attn_rows(const or_model* m, const layer_t* L, lstate_t* st, int64_t pos, const float* x, int R,
                      float* out) {
    const or_config* c = &m->c;
    const int nh = c->num_attention_heads, nkv = c->num_key_value_heads, hd = c->head_dim;
    float* qg = (float*)malloc((size_t)R * nh * 2 * hd * 4);
    float* kv = (float*)malloc((size_t)R * nkv * hd * 4);
    float* vv = (float*)malloc((size_t)R * nkv * hd * 4);
    float* res = (float*)malloc((size_t)R * nh * hd * 4);
    float* scores = (float*)malloc((size_t)nh * (pos + R) * 4);
    matvec_k(&L->q, x, R, qg);
    matvec_k(&L->k, x, R, kv);
    matvec_k(&L->v, x, R, vv);
    for (int r = 0; r < R; r++) {
        const int64_t p = pos + r;
        float* kr = kv + (int64_t)r * nkv * hd;
        for (int h = 0; h < nkv; h++) {
            converted_norm(kr + h * hd, L->k_norm, hd, c->rms_norm_eps);
            apply_rope(kr + h * hd, p, c->rotary_dim, c->rope_theta);
        }
        memcpy(st->keys + p * nkv * hd, kr, (size_t)nkv * hd * 4);
        memcpy(st->values + p * nkv * hd, vv + (int64_t)r * nkv * hd, (size_t)nkv * hd * 4);
        float* qr = qg + (int64_t)r * nh * 2 * hd;
        for (int h = 0; h < nh; h++) {
            float* q = qr + h * 2 * hd;
            converted_norm(q, L->q_norm, hd, c->rms_norm_eps);
            apply_rope(q, p, c->rotary_dim, c->rope_theta);
        }
        attend_row(qr, 2 * hd, hd, st->keys, st->values, nh, nkv, hd, p + 1, scores, res + (int64_t)r * nh * hd);
    }
    matvec_k(&L->o, res, R, out);
    free(qg); free(kv); free(vv); free(res); free(scores);
}

/* ----------------------------------------------------------------- MoE */
/* top_k_routes (moe.rs:21-54): softmax over the router logits (max, exp,
 * sum in expert order, divide), the top_k experts by probability (equal
 * probabilities rank the lower expert first; the reference's unstable sort
 * leaves that order unspecified), weights renormalized to sum to one when
 * norm_topk.  experts/weights receive topk entries; rank needs E ints. */
void or_route(const float* lg, int E, int topk, int norm_topk, int* rank, float* w) {
    float* pr = (float*)malloc((size_t)E * 4);
    float mx = -INFINITY;
    for (int e = 0; e < E; e++) mx = fmaxf(mx, lg[e]);
    float den = 0.f;
    for (int e = 0; e < E; e++) den += expf(lg[e] - mx);
    for (int e = 0; e < E; e++) pr[e] = expf(lg[e] - mx) / den;
    for (int e = 0; e < E; e++) rank[e] = e;
    for (int r = 0; r < topk; r++) {
        int best = r;
        for (int i = r + 1; i < E; i++)
            if (pr[rank[i]] > pr[rank[best]] || (pr[rank[i]] == pr[rank[best]] && rank[i] < rank[best])) best = i;
        int t = rank[r]; rank[r] = rank[best]; rank[best] = t;
    }
    float sum = 0.f;
    for (int r = 0; r < topk; r++) { w[r] = pr[rank[r]]; sum += w[r]; }
    if (norm_topk) for (int r = 0; r < topk; r++) w[r] /= sum;
    free(pr);
}
/* The sparse MoE block over R rows (quantized_moe.rs:237-460): router of
 * all rows, routes per row, then each distinct expert in ascending order
 * over the rows routed to it (routed_grouped_by_expert), the shared expert
 * over all rows; per row out = sum over its routes in route order of y * w,
 * then + shared * sigmoid(x . selector).  experts_out [R][topk] or NULL. */
static void moe_rows(const or_model* m, const layer_t* L, const float* x, int R, float* out, int* experts_out) {
    const or_config* c = &m->c;
    const int E = c->num_experts, H = c->hidden_size, F = c->moe_intermediate_size;
    const int Fs = c->shared_expert_intermediate_size, topk = c->num_experts_per_tok;
    const int FF = F > Fs ? F : Fs;
    float* lg = (float*)malloc((size_t)R * E * 4);
    int* rank = (int*)malloc((size_t)E * sizeof(int));
    int* route_e = (int*)malloc((size_t)R * topk * sizeof(int));
    float* route_w = (float*)malloc((size_t)R * topk * 4);
    float* yslot = (float*)malloc((size_t)R * topk * H * 4);
    float* xs = (float*)malloc((size_t)R * H * 4);
    float* g = (float*)malloc((size_t)R * FF * 4);
    float* u = (float*)malloc((size_t)R * FF * 4);
    float* y = (float*)malloc((size_t)R * H * 4);
    int* slot_of = (int*)malloc((size_t)R * topk * sizeof(int));
    matvec_k(&L->router, x, R, lg);
    for (int r = 0; r < R; r++) {
        or_route(lg + (int64_t)r * E, E, topk, c->norm_topk_prob, rank, route_w + r * topk);
        for (int q = 0; q < topk; q++) {
            route_e[r * topk + q] = rank[q];
            if (experts_out) experts_out[r * topk + q] = rank[q];
        }
    }
    /* the union's experts, one thread per expert (each expert's arithmetic is
     * the same whichever thread runs it; the products inside run serially) */
    int* used = (int*)malloc((size_t)E * sizeof(int));
    int nu = 0;
    for (int e = 0; e < E; e++)
        for (int i = 0; i < R * topk; i++)
            if (route_e[i] == e) { used[nu++] = e; break; }
#pragma omp parallel
    {
        float* txs = (float*)malloc((size_t)R * topk * H * 4);
        float* tg = (float*)malloc((size_t)R * topk * FF * 4);
        float* tu = (float*)malloc((size_t)R * topk * FF * 4);
        float* ty = (float*)malloc((size_t)R * topk * H * 4);
        int* tslot = (int*)malloc((size_t)R * topk * sizeof(int));
#pragma omp for schedule(dynamic, 1)
        for (int ui = 0; ui < nu; ui++) {
            const int e = used[ui];
            int n = 0;
            for (int r = 0; r < R; r++)
                for (int q = 0; q < topk; q++)
                    if (route_e[r * topk + q] == e) {
                        memcpy(txs + (int64_t)n * H, x + (int64_t)r * H, (size_t)H * 4);
                        tslot[n++] = r * topk + q;
                    }
            matvec_nk(&L->gate, L->gate.p + (int64_t)e * F * or_row_bytes(L->gate.dt, L->gate.cols), F, txs, n, tg, 1);
            matvec_nk(&L->up, L->up.p + (int64_t)e * F * or_row_bytes(L->up.dt, L->up.cols), F, txs, n, tu, 1);
            for (int i = 0; i < n * F; i++) tg[i] = (tg[i] / (1.f + expf(-tg[i]))) * tu[i];
            matvec_nk(&L->down, L->down.p + (int64_t)e * H * or_row_bytes(L->down.dt, L->down.cols), H, tg, n, ty, 1);
            for (int i = 0; i < n; i++) memcpy(yslot + (int64_t)tslot[i] * H, ty + (int64_t)i * H, (size_t)H * 4);
        }
        free(txs); free(tg); free(tu); free(ty); free(tslot);
    }
    free(used);
    for (int r = 0; r < R; r++) {
        float* o = out + (int64_t)r * H;
        for (int i = 0; i < H; i++) o[i] = 0.f;
        for (int q = 0; q < topk; q++) {
            const float* ys = yslot + (int64_t)(r * topk + q) * H;
            const float w = route_w[r * topk + q];
            for (int i = 0; i < H; i++) o[i] += ys[i] * w;
        }
    }
    matvec_nk(&L->sh_gate, L->sh_gate.p, Fs, x, R, g, 2);
    matvec_nk(&L->sh_up, L->sh_up.p, Fs, x, R, u, 2);
    for (int i = 0; i < R * Fs; i++) g[i] = (g[i] / (1.f + expf(-g[i]))) * u[i];
    matvec_nk(&L->sh_down, L->sh_down.p, H, g, R, y, 2);
    for (int r = 0; r < R; r++) {
        const float* xr = x + (int64_t)r * H;
        float sel = 0.f;
        for (int i = 0; i < H; i++) sel += xr[i] * L->selector[i];
        sel = 1.f / (1.f + expf(-sel));
        float* o = out + (int64_t)r * H;
        const float* ys = y + (int64_t)r * H;
        for (int i = 0; i < H; i++) o[i] = o[i] + ys[i] * sel;
    }
    free(lg); free(rank); free(route_e); free(route_w); free(yslot); free(xs); free(g); free(u); free(y); free(slot_of);
}

/* One decoder layer on R rows at positions pos.., in place
 * (quantized_layer.rs:101-225). */
static void layer_rows(const or_model* m, const layer_t* L, lstate_t* st, int64_t pos, float* h, int R,
                       int* experts) {
    const int H = m->c.hidden_size;
    float* xn = (float*)malloc((size_t)R * H * 4);
    float* mix = (float*)malloc((size_t)R * H * 4);
    for (int r = 0; r < R; r++) rms_norm(h + (int64_t)r * H, L->attn_norm, H, m->c.rms_norm_eps, xn + (int64_t)r * H);
    if (L->full) attn_rows(m, L, st, pos, xn, R, mix);
    else delta_rows(m, L, st, xn, R, mix);
    for (int i = 0; i < R * H; i++) h[i] = h[i] + mix[i];
    for (int r = 0; r < R; r++) rms_norm(h + (int64_t)r * H, L->post_norm, H, m->c.rms_norm_eps, xn + (int64_t)r * H);
    moe_rows(m, L, xn, R, mix, experts);
    for (int i = 0; i < R * H; i++) h[i] = h[i] + mix[i];
    free(xn); free(mix);
}
static void layer_row(const or_model* m, const layer_t* L, lstate_t* st, int64_t pos, float* h, int* experts) {
    layer_rows(m, L, st, pos, h, 1, experts);
}

/* Evaluate `rows` tokens (QuantizedModel::forward_detailed).  logits
 * [rows][vocab] and hidden [rows][hidden] (final-normed) may be NULL.
 * experts, when non-NULL, receives [rows][layers][topk] routed experts. */
int or_forward(const or_model* m, or_state* s, const uint32_t* tokens, int rows, float* logits, float* hidden,
               int32_t* experts) {
    const or_config* c = &m->c;
    const int H = c->hidden_size, topk = c->num_experts_per_tok;
    if (s->position + rows > s->max_pos) return -1;
    for (int r = 0; r < rows; r++)
        if (tokens[r] >= (uint32_t)c->vocab_size) return -2;
    /* passes of up to 8 rows through every layer (the reference's verify
     * width; a row's arithmetic does not depend on the pass it runs in) */
    if (s->snap_rows > 0 && rows > s->snap_rows) return -3;
    s->snap_pos0 = s->position;
    s->snap_taken = rows;
    /* order 2 restates the wide pass: from 64 rows, passes of up to 512 */
    const int pass = (g_order == 2 && rows >= 64) ? 512 : 8;
    for (int r0 = 0; r0 < rows; r0 += pass) {
        const int R = rows - r0 < pass ? rows - r0 : pass;
        float* h = (float*)malloc((size_t)R * H * 4);
        float* hn = (float*)malloc((size_t)R * H * 4);
        int* ex = (int*)malloc((size_t)R * topk * sizeof(int));
        for (int r = 0; r < R; r++)
            or_dequant_rows(m->embed.dt, m->embed.p + (int64_t)tokens[r0 + r] * or_row_bytes(m->embed.dt, H), 1, H,
                            h + (int64_t)r * H);
        for (int l = 0; l < c->num_hidden_layers; l++) {
            layer_rows(m, &m->layers[l], &s->l[l], s->position, h, R, ex);
            if (experts)
                for (int r = 0; r < R; r++)
                    for (int i = 0; i < topk; i++)
                        experts[((int64_t)(r0 + r) * c->num_hidden_layers + l) * topk + i] = ex[r * topk + i];
        }
        for (int r = 0; r < R; r++) rms_norm(h + (int64_t)r * H, m->out_norm, H, c->rms_norm_eps, hn + (int64_t)r * H);
        if (hidden) memcpy(hidden + (int64_t)r0 * H, hn, (size_t)R * H * 4);
        if (logits) matvec_k(&m->lm_head, hn, R, logits + (int64_t)r0 * c->vocab_size);
        s->position += R;
        free(h); free(hn); free(ex);
    }
    return 0;
}

/* One MTP predictor step (quantized_mtp.rs:175-227): token + previous
 * hidden row -> next hidden row and logits over the first head_rows rows
 * of the LM head (0 = no logits). */
int or_mtp_forward(const or_model* m, or_state* s, uint32_t token, const float* hidden_in, int64_t head_rows,
                   float* logits, float* hidden_out) {
    const or_config* c = &m->c;
    const int H = c->hidden_size;
    if (!m->has_mtp) return -1;
    float* e = (float*)malloc((size_t)2 * H * 4);
    float* tmp = (float*)malloc((size_t)H * 4);
    float* h = (float*)malloc((size_t)H * 4);
    or_dequant_rows(m->embed.dt, m->embed.p + (int64_t)token * or_row_bytes(m->embed.dt, H), 1, H, tmp);
    rms_norm(tmp, m->enorm, H, c->rms_norm_eps, e);
    rms_norm(hidden_in, m->hnorm, H, c->rms_norm_eps, e + H);
    matvec(&m->eh_proj, e, h);
    layer_row(m, &m->mtp, &s->mtp, s->mtp_position, h, NULL);
    rms_norm(h, m->head_norm, H, c->rms_norm_eps, tmp);
    if (hidden_out) memcpy(hidden_out, tmp, (size_t)H * 4);
    if (logits && head_rows > 0) matvec_n(&m->lm_head, m->lm_head.p, head_rows, tmp, logits, 0);
    s->mtp_position++;
    free(e); free(tmp); free(h);
    return 0;
}

void or_state_set_mtp_position(or_state* s, int64_t p) { s->mtp_position = p; }

/* ------------------------------------------------------------ state images
 * The library's state-image layout (iq.h, iq_state_export), restated so a
 * test can start the oracle from exactly the state the device holds
 * (teacher forcing) and compare the states after a step: a 56-byte header
 * {magic "IQSTATE1", i32 version, i32 layers, i64 position, i64 mtp_position,
 * i32 has_mtp, kv_dim, conv_dim, conv_taps, rec_size, pad}, then per decoder
 * layer the KV rows (keys then values, [pos][kv_dim]) of an attention layer
 * or the conv [conv_dim][taps] and recurrent [nv][dk][dv] state of a
 * DeltaNet layer, then the MTP block's KV rows; all f32.  The reference's
 * own image (QuantizedStateImage, src/qwen/quantized_model.rs:59-100) holds
 * the same per-layer tensors. */
typedef struct {
    char magic[8];
    int32_t version, layers;
    int64_t position, mtp_position;
    int32_t has_mtp, kv_dim, conv_dim, conv_taps, rec_size, pad;
} img_header_t;

static void img_dims(const or_model* m, int64_t* kv_dim, int64_t* conv_n, int64_t* rec_n) {
    const or_config* c = &m->c;
    *kv_dim = (int64_t)c->num_key_value_heads * c->head_dim;
    int64_t conv_dim = 2 * (int64_t)c->linear_num_key_heads * c->linear_key_head_dim +
                       (int64_t)c->linear_num_value_heads * c->linear_value_head_dim;
    *conv_n = conv_dim * (c->linear_conv_kernel_dim - 1);
    *rec_n = (int64_t)c->linear_num_value_heads * c->linear_key_head_dim * c->linear_value_head_dim;
}

static int64_t img_bytes(const or_model* m, int64_t pos, int64_t mtp_pos) {
    int64_t kv, cn, rn;
    img_dims(m, &kv, &cn, &rn);
    int64_t b = (int64_t)sizeof(img_header_t);
    for (int l = 0; l < m->c.num_hidden_layers; l++) b += m->layers[l].full ? 2 * pos * kv * 4 : (cn + rn) * 4;
    if (m->has_mtp) b += 2 * mtp_pos * kv * 4;
    return b;
}

int64_t or_state_image_size(const or_model* m, const or_state* s) {
    return img_bytes(m, s->position, m->has_mtp ? s->mtp_position : 0);
}

int or_state_export(const or_model* m, const or_state* s, uint8_t* out, int64_t bytes) {
    int64_t kv, cn, rn;
    img_dims(m, &kv, &cn, &rn);
    const int64_t mtp_pos = m->has_mtp ? s->mtp_position : 0;
    if (bytes < img_bytes(m, s->position, mtp_pos)) return -1;
    img_header_t h;
    memset(&h, 0, sizeof h);
    memcpy(h.magic, "IQSTATE1", 8);
    h.version = 1;
    h.layers = m->c.num_hidden_layers;
    h.position = s->position;
    h.mtp_position = mtp_pos;
    h.has_mtp = m->has_mtp;
    h.kv_dim = (int32_t)kv;
    h.conv_dim = (int32_t)(2 * (int64_t)m->c.linear_num_key_heads * m->c.linear_key_head_dim +
                           (int64_t)m->c.linear_num_value_heads * m->c.linear_value_head_dim);
    h.conv_taps = m->c.linear_conv_kernel_dim - 1;
    h.rec_size = (int32_t)rn;
    memcpy(out, &h, sizeof h);
    uint8_t* p = out + sizeof h;
    for (int l = 0; l < m->c.num_hidden_layers; l++) {
        const lstate_t* st = &s->l[l];
        if (m->layers[l].full) {
            size_t n = (size_t)(s->position * kv * 4);
            memcpy(p, st->keys, n); memcpy(p + n, st->values, n); p += 2 * n;
        } else {
            memcpy(p, st->conv, (size_t)cn * 4); memcpy(p + cn * 4, st->rec, (size_t)rn * 4); p += (cn + rn) * 4;
        }
    }
    if (m->has_mtp) {
        size_t n = (size_t)(mtp_pos * kv * 4);
        memcpy(p, s->mtp.keys, n); memcpy(p + n, s->mtp.values, n);
    }
    return 0;
}

int or_state_import(const or_model* m, or_state* s, const uint8_t* in, int64_t bytes) {
    img_header_t h;
    int64_t kv, cn, rn;
    img_dims(m, &kv, &cn, &rn);
    if (bytes < (int64_t)sizeof h) return -1;
    memcpy(&h, in, sizeof h);
    if (memcmp(h.magic, "IQSTATE1", 8) || h.version != 1 || h.layers != m->c.num_hidden_layers) return -2;
    if (h.kv_dim != kv || h.rec_size != rn || h.has_mtp != m->has_mtp) return -3;
    if (h.position > s->max_pos || h.mtp_position > s->max_pos) return -4;
    if (bytes != img_bytes(m, h.position, h.mtp_position)) return -5;
    const uint8_t* p = in + sizeof h;
    for (int l = 0; l < m->c.num_hidden_layers; l++) {
        lstate_t* st = &s->l[l];
        if (m->layers[l].full) {
            size_t n = (size_t)(h.position * kv * 4);
            memcpy(st->keys, p, n); memcpy(st->values, p + n, n); p += 2 * n;
        } else {
            memcpy(st->conv, p, (size_t)cn * 4); memcpy(st->rec, p + cn * 4, (size_t)rn * 4); p += (cn + rn) * 4;
        }
    }
    if (m->has_mtp) {
        size_t n = (size_t)(h.mtp_position * kv * 4);
        memcpy(s->mtp.keys, p, n); memcpy(s->mtp.values, p + n, n);
    }
    s->position = h.position;
    s->mtp_position = h.mtp_position;
    return 0;
}
