/*
 * vtx_ref.c — CPU ORACLE for the voxtral.cpp attention node.  TEST
 * INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg call it as the checker.  The product (voxtral.cpp_b200) never
 * links or calls it.
 *
 * It restates the arithmetic of ggml's CPU GGML_OP_FLASH_ATTN_EXT kernel,
 * ggml_compute_forward_flash_attn_ext_f16 in ggml/src/ggml-cpu/ops.cpp at
 * ggml-org/ggml@5cecdad692d868e28dbd2f7c468504770108f30c — the revision the
 * reference pins with FetchContent (reference CMakeLists.txt:33-41).  That
 * source is NOT present next to the reference, so the restatement follows
 * ggml's published algorithm (one output row per (query, head); online
 * softmax over keys with running max M and sum S; masked keys skipped):
 *
 *   - Q is first converted to K's vec_dot type: F16 when K is F16 (Q rounded
 *     to half), Q8_0 when K is Q8_0 (Q quantized per 32-block, int8 dot with
 *     per-block scales), F32 when K is F32.
 *   - s = dot(Q, K_j) * scale; with logit_softcap: scale /= softcap first and
 *     s = softcap * tanhf(s); then s += slope * mask[i, j]; mask == -inf
 *     skips key j entirely.
 *   - V accumulator VKQ is HALF precision when V is F16 (every rescale
 *     VKQ *= expf(Mold - M) and every update VKQ = fma(v, expf(s - M), VKQ)
 *     rounds to half), F32 otherwise (V converted to F32 first).
 *   - out = VKQ / S, or 0 when S == 0 (every key masked).
 *   - ALiBi slope: max_bias > 0 ? (h < n_head_log2 ? m0^(h+1)
 *     : m1^(2(h - n_head_log2) + 1)) : 1, n_head_log2 = 2^floor(log2(Hq)).
 *
 * Mode VTX_REF_FP64 is an independent "truth": the same masked softmax in
 * double precision on the exact input values (Q not rounded, K/V dequantized
 * exactly), one pass with the true maximum.
 *
 * Which reference lines the geometry follows:
 *   views and GQA broadcast   src/voxtral.cpp:1589-1611, 1783-1802
 *   mask values               src/voxtral.cpp:2103-2111 (causal),
 *                             src/voxtral.cpp:2181-2188 (window 750)
 *   KV cache layout           src/voxtral.cpp:1126-1136, 1755-1781
 *
 * Parity status: the op-level arithmetic is UNPINNED against ggml itself
 * (no ggml source or binary exists in this environment and the reference's
 * own tests pin only end-to-end logits that need absent model weights).  The
 * pieces that can be pinned are: the Q8_0 block format and quantizer against
 * gguf-py 0.19.0 (gguf/quants.py, ggml's Python port), the half conversions
 * against numpy, and the fp64 mode against torch float64 attention; see
 * tests/golden/make_golden.py.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/vtx_fa.h"

#define VTX_REF_GGML 0
#define VTX_REF_FP64 1

typedef _Float16 f16;

static inline float h2f(uint16_t h) { f16 x; memcpy(&x, &h, 2); return (float)x; }
static inline uint16_t f2h(float f) { f16 x = (f16)f; uint16_t h; memcpy(&h, &x, 2); return h; }

/* ---- Q8_0 ------------------------------------------------------------- */

/* ggml quantize_row_q8_0_ref (ggml/src/ggml-quants.c): d = amax/127,
 * id = 1/d, q = roundf(x*id) (ties away from zero).  Used to build Q8_0 KV
 * caches; pinned against gguf-py's Q8_0.quantize_blocks. */
void vtx_ref_quantize_q8_0(const float *x, vtx_block_q8_0 *y, int64_t n)
{
    const int64_t nb = n / VTX_QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        float amax = 0.0f;
        for (int j = 0; j < VTX_QK8_0; j++) {
            const float v = fabsf(x[i * VTX_QK8_0 + j]);
            if (v > amax) amax = v;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = f2h(d);
        for (int j = 0; j < VTX_QK8_0; j++) {
            y[i].qs[j] = (int8_t)roundf(x[i * VTX_QK8_0 + j] * id);
        }
    }
}

/* The x86 SIMD from_float of ggml-cpu (quantize_row_q8_0 with AVX2):
 * d = amax/127, id = 127/amax, q = round-half-even(x*id).  ggml's CPU
 * flash attention quantizes each Q row with this before the Q8_0 dot. */
void vtx_ref_quantize_q8_0_rne(const float *x, vtx_block_q8_0 *y, int64_t n)
{
    const int64_t nb = n / VTX_QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        float amax = 0.0f;
        for (int j = 0; j < VTX_QK8_0; j++) {
            const float v = fabsf(x[i * VTX_QK8_0 + j]);
            if (v > amax) amax = v;
        }
        const float d = amax / 127.0f;
        const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
        y[i].d = f2h(d);
        for (int j = 0; j < VTX_QK8_0; j++) {
            y[i].qs[j] = (int8_t)nearbyintf(x[i * VTX_QK8_0 + j] * id);
        }
    }
}

void vtx_ref_dequantize_q8_0(const vtx_block_q8_0 *x, float *y, int64_t n)
{
    const int64_t nb = n / VTX_QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        const float d = h2f(x[i].d);
        for (int j = 0; j < VTX_QK8_0; j++) y[i * VTX_QK8_0 + j] = d * (float)x[i].qs[j];
    }
}

void vtx_ref_f32_to_f16(const float *x, uint16_t *y, int64_t n)
{
    for (int64_t i = 0; i < n; i++) y[i] = f2h(x[i]);
}

void vtx_ref_f16_to_f32(const uint16_t *x, float *y, int64_t n)
{
    for (int64_t i = 0; i < n; i++) y[i] = h2f(x[i]);
}

/* ---- attention -------------------------------------------------------- */

typedef struct {
    const vtx_tensor *q, *k, *v, *mask;
    const vtx_fa_params *p;
    vtx_tensor *dst;
    int mode;
    int64_t n_rows;
    atomic_long next;
    float m0, m1;
    uint32_t n_head_log2;
    float scale;
} job_t;

static inline int tensor_elem_size(int type) { return type == VTX_TYPE_F32 ? 4 : 2; }

/* Dot of an f32 vector with an F16 row, f32 lanes like ggml_vec_dot_f16. */
static inline float dot_f16(const float *a, const uint16_t *b, int64_t n)
{
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t i = 0;
    for (; i + 8 <= n; i += 8) {
        for (int l = 0; l < 8; l++) {
            f16 h; memcpy(&h, &b[i + l], 2);
            acc[l] = fmaf(a[i + l], (float)h, acc[l]);
        }
    }
    float s = 0.0f;
    for (int l = 0; l < 8; l++) s += acc[l];
    for (; i < n; i++) s += a[i] * h2f(b[i]);
    return s;
}

static inline float dot_f32(const float *a, const float *b, int64_t n)
{
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s = 0.0f;
    for (int l = 0; l < 8; l++) s += acc[l];
    for (; i < n; i++) s += a[i] * b[i];
    return s;
}

/* ggml_vec_dot_q8_0_q8_0: per block, integer dot times d_x*d_y, f32 sum. */
static inline float dot_q8_0(const vtx_block_q8_0 *x, const vtx_block_q8_0 *y, int64_t n)
{
    float s = 0.0f;
    for (int64_t b = 0; b < n / VTX_QK8_0; b++) {
        int32_t isum = 0;
        for (int j = 0; j < VTX_QK8_0; j++) isum += (int32_t)x[b].qs[j] * (int32_t)y[b].qs[j];
        s = fmaf(h2f(x[b].d) * h2f(y[b].d), (float)isum, s);
    }
    return s;
}

/* Structural mask from params: 0 allowed, -inf masked.  Equivalent to the
 * host-built masks of src/voxtral.cpp:2103-2111 and :2181-2188. */
static inline int structurally_masked(const vtx_fa_params *p, int64_t iq, int64_t ik,
                                      int64_t n_q, int64_t n_kv)
{
    if (!p->causal) return 0;
    const int64_t pos = iq + (n_kv - n_q);
    if (ik > pos) return 1;
    if (p->window > 0 && ik < pos - (p->window - 1)) return 1;
    return 0;
}

static float row_slope(const job_t *J, int64_t h)
{
    if (!(J->p->max_bias > 0.0f)) return 1.0f;
    return h < (int64_t)J->n_head_log2 ? powf(J->m0, (float)(h + 1))
                                       : powf(J->m1, (float)(2 * (h - J->n_head_log2) + 1));
}

static void row_ggml(job_t *J, int64_t iq1, int64_t iq2, int64_t iq3, void *scratch)
{
    const vtx_tensor *q = J->q, *k = J->k, *v = J->v, *mask = J->mask;
    const int64_t DK = k->ne[0], DV = v->ne[0], n_kv = k->ne[1], n_q = q->ne[1];
    const int64_t ik2 = iq2 / (q->ne[2] / k->ne[2]), ik3 = iq3 / (q->ne[3] / k->ne[3]);
    const int64_t iv2 = iq2 / (q->ne[2] / v->ne[2]), iv3 = iq3 / (q->ne[3] / v->ne[3]);
    const float slope = row_slope(J, iq2);
    const float softcap = J->p->logit_softcap;
    const float scale = J->scale;

    float *qf = (float *)scratch;                 /* DK: Q as f32 (rounded to half for F16 K) */
    float *vkq32 = qf + DK;                       /* DV */
    float *v32 = vkq32 + DV;                      /* DV */
    uint16_t *vkq16 = (uint16_t *)(v32 + DV);     /* DV */
    vtx_block_q8_0 *qq = (vtx_block_q8_0 *)(vkq16 + DV + 8);

    const char *pq = (const char *)q->data + iq1 * q->nb[1] + iq2 * q->nb[2] + iq3 * q->nb[3];
    for (int64_t d = 0; d < DK; d++) {
        float x = q->type == VTX_TYPE_F32 ? ((const float *)pq)[d] : h2f(((const uint16_t *)pq)[d]);
        qf[d] = x;
    }
    if (k->type == VTX_TYPE_F16) {
        for (int64_t d = 0; d < DK; d++) qf[d] = h2f(f2h(qf[d]));
    } else if (k->type == VTX_TYPE_Q8_0) {
        vtx_ref_quantize_q8_0_rne(qf, qq, DK);
    }

    const uint16_t *mp = mask ? (const uint16_t *)((const char *)mask->data + iq1 * mask->nb[1] +
                                                   (iq2 % mask->ne[2]) * mask->nb[2] +
                                                   (iq3 % mask->ne[3]) * mask->nb[3])
                              : NULL;

    float S = 0.0f, M = -INFINITY;
    const int vf16 = v->type == VTX_TYPE_F16;
    if (vf16) memset(vkq16, 0, DV * 2);
    else memset(vkq32, 0, DV * 4);

    for (int64_t ic = 0; ic < n_kv; ic++) {
        if (structurally_masked(J->p, iq1, ic, n_q, n_kv)) continue;
        const float mv = mp ? slope * h2f(*(const uint16_t *)((const char *)mp + ic * mask->nb[0])) : 0.0f;
        if (mv == -INFINITY) continue;

        const char *kd = (const char *)k->data + ic * k->nb[1] + ik2 * k->nb[2] + ik3 * k->nb[3];
        float s;
        if (k->type == VTX_TYPE_F16) s = dot_f16(qf, (const uint16_t *)kd, DK);
        else if (k->type == VTX_TYPE_F32) s = dot_f32(qf, (const float *)kd, DK);
        else s = dot_q8_0((const vtx_block_q8_0 *)kd, qq, DK);

        s = s * scale;
        if (softcap != 0.0f) s = softcap * tanhf(s);
        s += mv;

        const float Mold = M;
        float ms = 1.0f, vs = 1.0f;
        const char *vd = (const char *)v->data + ic * v->nb[1] + iv2 * v->nb[2] + iv3 * v->nb[3];
        if (vf16) {
            if (s > M) {
                M = s;
                ms = expf(Mold - M);
                for (int64_t d = 0; d < DV; d++) vkq16[d] = f2h(h2f(vkq16[d]) * ms);
            } else {
                vs = expf(s - M);
            }
            const uint16_t *vh = (const uint16_t *)vd;
            for (int64_t d = 0; d < DV; d++) vkq16[d] = f2h(fmaf(h2f(vh[d]), vs, h2f(vkq16[d])));
        } else {
            if (s > M) {
                M = s;
                ms = expf(Mold - M);
                for (int64_t d = 0; d < DV; d++) vkq32[d] *= ms;
            } else {
                vs = expf(s - M);
            }
            const float *vrow;
            if (v->type == VTX_TYPE_Q8_0) {
                vtx_ref_dequantize_q8_0((const vtx_block_q8_0 *)vd, v32, DV);
                vrow = v32;
            } else {
                vrow = (const float *)vd;
            }
            for (int64_t d = 0; d < DV; d++) vkq32[d] = fmaf(vrow[d], vs, vkq32[d]);
        }
        S = S * ms + vs;
    }
    if (vf16)
        for (int64_t d = 0; d < DV; d++) vkq32[d] = h2f(vkq16[d]);
    const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;

    float *out = (float *)((char *)J->dst->data + iq1 * J->dst->nb[2] + iq2 * J->dst->nb[1] +
                           iq3 * J->dst->nb[3]);
    for (int64_t d = 0; d < DV; d++) out[d] = vkq32[d] * S_inv;
}

static double load_elem_f64(const vtx_tensor *t, const char *row, int64_t d)
{
    if (t->type == VTX_TYPE_F32) return ((const float *)row)[d];
    if (t->type == VTX_TYPE_F16) return h2f(((const uint16_t *)row)[d]);
    const vtx_block_q8_0 *b = (const vtx_block_q8_0 *)row + d / VTX_QK8_0;
    return (double)h2f(b->d) * (double)b->qs[d % VTX_QK8_0];
}

static void row_fp64(job_t *J, int64_t iq1, int64_t iq2, int64_t iq3, void *scratch)
{
    const vtx_tensor *q = J->q, *k = J->k, *v = J->v, *mask = J->mask;
    const int64_t DK = k->ne[0], DV = v->ne[0], n_kv = k->ne[1], n_q = q->ne[1];
    const int64_t ik2 = iq2 / (q->ne[2] / k->ne[2]), ik3 = iq3 / (q->ne[3] / k->ne[3]);
    const int64_t iv2 = iq2 / (q->ne[2] / v->ne[2]), iv3 = iq3 / (q->ne[3] / v->ne[3]);
    const double slope = row_slope(J, iq2);
    const double softcap = J->p->logit_softcap;
    double scale = J->p->scale;
    if (softcap != 0.0) scale /= softcap;

    double *qd = (double *)scratch;
    double *sc = qd + DK;          /* n_kv scores */
    double *acc = sc + n_kv;       /* DV */
    const char *pq = (const char *)q->data + iq1 * q->nb[1] + iq2 * q->nb[2] + iq3 * q->nb[3];
    for (int64_t d = 0; d < DK; d++) qd[d] = load_elem_f64(q, pq, d);

    const uint16_t *mp = mask ? (const uint16_t *)((const char *)mask->data + iq1 * mask->nb[1] +
                                                   (iq2 % mask->ne[2]) * mask->nb[2] +
                                                   (iq3 % mask->ne[3]) * mask->nb[3])
                              : NULL;
    double M = -INFINITY;
    for (int64_t ic = 0; ic < n_kv; ic++) {
        sc[ic] = -INFINITY;
        if (structurally_masked(J->p, iq1, ic, n_q, n_kv)) continue;
        const double mv = mp ? slope * (double)h2f(*(const uint16_t *)((const char *)mp + ic * mask->nb[0])) : 0.0;
        if (mv == -INFINITY) continue;
        const char *kd = (const char *)k->data + ic * k->nb[1] + ik2 * k->nb[2] + ik3 * k->nb[3];
        double s = 0.0;
        for (int64_t d = 0; d < DK; d++) s += qd[d] * load_elem_f64(k, kd, d);
        s *= scale;
        if (softcap != 0.0) s = softcap * tanh(s);
        s += mv;
        sc[ic] = s;
        if (s > M) M = s;
    }
    for (int64_t d = 0; d < DV; d++) acc[d] = 0.0;
    double S = 0.0;
    if (M != -INFINITY) {
        for (int64_t ic = 0; ic < n_kv; ic++) {
            if (sc[ic] == -INFINITY) continue;
            const double w = exp(sc[ic] - M);
            S += w;
            const char *vd = (const char *)v->data + ic * v->nb[1] + iv2 * v->nb[2] + iv3 * v->nb[3];
            for (int64_t d = 0; d < DV; d++) acc[d] += w * load_elem_f64(v, vd, d);
        }
    }
    float *out = (float *)((char *)J->dst->data + iq1 * J->dst->nb[2] + iq2 * J->dst->nb[1] +
                           iq3 * J->dst->nb[3]);
    for (int64_t d = 0; d < DV; d++) out[d] = S == 0.0 ? 0.0f : (float)(acc[d] / S);
}

static void *worker(void *arg)
{
    job_t *J = (job_t *)arg;
    const int64_t DK = J->k->ne[0], DV = J->v->ne[0], n_kv = J->k->ne[1];
    const size_t bytes = J->mode == VTX_REF_FP64 ? (size_t)(DK + n_kv + DV + 8) * sizeof(double)
                                                 : (size_t)(DK + 3 * DV + 64) * sizeof(float) + DK * 2;
    void *scratch = malloc(bytes);
    if (!scratch) return NULL;
    const int64_t nq1 = J->q->ne[1], nq2 = J->q->ne[2];
    for (;;) {
        const long r = atomic_fetch_add(&J->next, 1);
        if (r >= J->n_rows) break;
        const int64_t iq3 = r / (nq2 * nq1);
        const int64_t iq2 = (r - iq3 * nq2 * nq1) / nq1;
        const int64_t iq1 = r - iq3 * nq2 * nq1 - iq2 * nq1;
        if (J->mode == VTX_REF_FP64) row_fp64(J, iq1, iq2, iq3, scratch);
        else row_ggml(J, iq1, iq2, iq3, scratch);
    }
    free(scratch);
    return NULL;
}

/* Returns 0 on success, a negative vtx_status otherwise.  All pointers are
 * host pointers.  Rows (query, head, batch) are spread over n_threads. */
int vtx_ref_flash_attn_ext(const vtx_tensor *q, const vtx_tensor *k, const vtx_tensor *v,
                           const vtx_tensor *mask, const vtx_fa_params *p, vtx_tensor *dst,
                           int mode, int n_threads)
{
    if (!q || !k || !v || !p || !dst) return VTX_ERR_NULL;
    if (k->ne[1] != v->ne[1] || k->ne[2] != v->ne[2] || q->ne[0] != k->ne[0]) return VTX_ERR_SHAPE;
    if (k->ne[2] <= 0 || q->ne[2] % k->ne[2] != 0 || q->ne[3] % k->ne[3] != 0) return VTX_ERR_SHAPE;
    if (k->type == VTX_TYPE_Q8_0 && k->ne[0] % VTX_QK8_0) return VTX_ERR_SHAPE;
    if (dst->ne[0] != v->ne[0] || dst->ne[1] != q->ne[2] || dst->ne[2] != q->ne[1]) return VTX_ERR_SHAPE;
    if (mask && (mask->type != VTX_TYPE_F16 || mask->ne[0] < k->ne[1] || mask->ne[1] < q->ne[1]))
        return VTX_ERR_SHAPE;

    job_t J;
    memset(&J, 0, sizeof(J));
    J.q = q; J.k = k; J.v = v; J.mask = mask; J.p = p; J.dst = dst; J.mode = mode;
    J.n_rows = q->ne[1] * q->ne[2] * q->ne[3];
    atomic_init(&J.next, 0);
    const uint32_t n_head = (uint32_t)q->ne[2];
    J.n_head_log2 = 1u << (uint32_t)floor(log2((double)n_head));
    J.m0 = powf(2.0f, -(p->max_bias) / J.n_head_log2);
    J.m1 = powf(2.0f, -(p->max_bias / 2.0f) / J.n_head_log2);
    J.scale = p->scale;
    if (p->logit_softcap != 0.0f) J.scale /= p->logit_softcap;

    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (J.n_rows < n_threads) n_threads = (int)(J.n_rows > 0 ? J.n_rows : 1);
    pthread_t th[256];
    int started = 0;
    for (int t = 1; t < n_threads; t++)
        if (pthread_create(&th[started], NULL, worker, &J) == 0) started++;
    worker(&J);
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return 0;
}

/* Ragged batched decode on the host, same contract as
 * vtx_flash_attn_decode_batched but with host pointers. */
int vtx_ref_decode_batched(const vtx_decode_batch *b, int mode, int n_threads)
{
    if (!b || !b->q || !b->k_ptrs || !b->v_ptrs || !b->kv_len || !b->dst) return VTX_ERR_NULL;
    const int D = b->head_dim;
    const size_t esz = b->kv_type == VTX_TYPE_F32 ? 4 : 2;
    for (int s = 0; s < b->n_seq; s++) {
        vtx_tensor q = {VTX_TYPE_F32, 0, {D, 1, b->n_head_q, 1}, {4, 4 * (size_t)D * b->n_head_q, 4 * (size_t)D, 0}, 0};
        q.data = (void *)(b->q + (size_t)s * b->n_head_q * D);
        q.nb[3] = q.nb[2] * b->n_head_q;
        vtx_tensor k = {b->kv_type, 0, {D, b->kv_len[s], b->n_head_kv, 1}, {0, b->kv_nb1, b->kv_nb2, 0}, 0};
        k.nb[0] = b->kv_type == VTX_TYPE_Q8_0 ? sizeof(vtx_block_q8_0) : esz;
        k.nb[3] = b->kv_nb2 * b->n_head_kv;
        k.data = (void *)b->k_ptrs[s];
        vtx_tensor v = k;
        v.data = (void *)b->v_ptrs[s];
        vtx_tensor o = {VTX_TYPE_F32, 0, {D, b->n_head_q, 1, 1}, {4, 4 * (size_t)D, 4 * (size_t)D * b->n_head_q, 0}, 0};
        o.nb[3] = o.nb[2];
        o.data = b->dst + (size_t)s * b->n_head_q * D;
        vtx_fa_params p;
        memset(&p, 0, sizeof(p));
        p.scale = b->scale;
        int rc = vtx_ref_flash_attn_ext(&q, &k, &v, NULL, &p, &o, mode, n_threads);
        if (rc) return rc;
    }
    return 0;
}

/* ---- KV append: RoPE + cache write (decoder layer) -------------------------
 * Restates the decoder layer's cache update (src/voxtral.cpp:1744-1770):
 *   q = ggml_rope_ext(q, positions, NULL, head_dim, mode 0, n_ctx_orig 0,
 *                     freq_base, freq_scale 1, ext_factor 0, attn_factor 1,
 *                     beta_fast 0, beta_slow 0);   k = the same;
 *   ggml_cpy(k -> K cache row kv_offset + i), ggml_cpy(v -> V cache row).
 * ggml's CPU rope for mode 0 ("normal": adjacent pairs (x[2i], x[2i+1])) as
 * published (ggml_rope_cache_init / rope_yarn in ggml-cpu/ops.cpp): one float
 * theta per token, starting at (float)pos and multiplied by
 * theta_scale = powf(freq_base, -2/n_dims) after each pair; per pair
 * c = cosf(theta), s = sinf(theta); y0 = x0*c - x1*s, y1 = x0*s + x1*c.
 * The cache write converts each float row to the cache type: F32 unchanged,
 * F16 round-to-nearest-even, Q8_0 with the CPU from_float (quantize_q8_0_rne).
 * slots[i] is the cache row of token i; the build replaces the reference's
 * shift-left memmove (src/voxtral.cpp:1237-1266) by a ring slot, which keeps
 * the same set of rows.
 * Mode VTX_REF_FP64: theta_i = pos * freq_base^(-2i/n_dims) and cos/sin in
 * double (an independent truth for the rotation; cache writes as above).
 * q, k, v, q_out are contiguous [n_tokens][n_head][head_dim] floats. */
static void rope_row(const float *x, float *y, int D, int32_t pos, float theta_scale, double freq_base, int mode)
{
    float theta = (float)pos;
    for (int i = 0; i < D / 2; i++) {
        float c, s;
        if (mode == VTX_REF_FP64) {
            const double th = (double)pos * pow(freq_base, -2.0 * i / D);
            c = (float)cos(th);
            s = (float)sin(th);
        } else {
            c = cosf(theta);
            s = sinf(theta);
            theta *= theta_scale;
        }
        const float x0 = x[2 * i], x1 = x[2 * i + 1];
        y[2 * i] = x0 * c - x1 * s;
        y[2 * i + 1] = x0 * s + x1 * c;
    }
}

static void cache_store(const float *x, void *dst, int D, int kv_type)
{
    if (kv_type == VTX_TYPE_F32) memcpy(dst, x, (size_t)D * 4);
    else if (kv_type == VTX_TYPE_F16) vtx_ref_f32_to_f16(x, (uint16_t *)dst, D);
    else vtx_ref_quantize_q8_0_rne(x, (vtx_block_q8_0 *)dst, D);
}

int vtx_ref_kv_append(int n_tokens, int n_head_q, int n_head_kv, int head_dim, int kv_type, float freq_base,
                      const float *q, float *q_out, const float *k, const float *v, const int32_t *positions,
                      const int32_t *slots, void *k_cache, void *v_cache, size_t cache_nb1, int mode)
{
    if (!k || !v || !positions || !slots || !k_cache || !v_cache) return VTX_ERR_NULL;
    if (head_dim % 32 || head_dim <= 0) return VTX_ERR_UNSUPPORTED;
    const int D = head_dim;
    const float theta_scale = powf(freq_base, -2.0f / (float)D);
    const size_t head_bytes = kv_type == VTX_TYPE_F32 ? (size_t)D * 4
                            : kv_type == VTX_TYPE_F16 ? (size_t)D * 2 : (size_t)D / 32 * sizeof(vtx_block_q8_0);
    float *tmp = (float *)malloc((size_t)D * sizeof(float));
    if (!tmp) return VTX_ERR_CUDA;
    for (int t = 0; t < n_tokens; t++) {
        if (q && q_out)
            for (int h = 0; h < n_head_q; h++)
                rope_row(q + ((size_t)t * n_head_q + h) * D, q_out + ((size_t)t * n_head_q + h) * D, D,
                         positions[t], theta_scale, freq_base, mode);
        char *krow = (char *)k_cache + (size_t)slots[t] * cache_nb1;
        char *vrow = (char *)v_cache + (size_t)slots[t] * cache_nb1;
        for (int h = 0; h < n_head_kv; h++) {
            rope_row(k + ((size_t)t * n_head_kv + h) * D, tmp, D, positions[t], theta_scale, freq_base, mode);
            cache_store(tmp, krow + h * head_bytes, D, kv_type);
            cache_store(v + ((size_t)t * n_head_kv + h) * D, vrow + h * head_bytes, D, kv_type);
        }
    }
    free(tmp);
    return 0;
}

/* ---- attention output projection ----------------------------------------
 * dst[t][n] = residual[t][n] + bias[n] + sum_k A[t][k] * W[n][k]: the
 * ggml_mul_mat(attn_o_weight, attn_out) (+ attn_o_bias) + residual add after
 * each attention node (src/voxtral.cpp:1612-1617 encoder, :1804-1809
 * decoder).  ggml mode: ggml's CPU mul_mat for an F16 weight converts the F32
 * activations to its vec_dot type, F16 (round to nearest even), and
 * accumulates the F16 x F16 products in f32 (ggml_vec_dot_f16); the bias and
 * residual adds are f32.  fp64 mode: A unrounded, everything in double.
 * A: n rows of K floats at a stride of lda floats; W: N rows of K halves at
 * ldw; residual / dst: n rows of N floats at ldr / ldd (residual may be
 * NULL, and may equal dst); bias: N floats or NULL.  Rows are spread over
 * n_threads. */
typedef struct {
    const float *A; int64_t lda;
    const uint16_t *W; int64_t ldw;
    const float *bias, *res; int64_t ldr;
    float *dst; int64_t ldd;
    int n, K, N, mode;
    atomic_long next;
} proj_job_t;

static void *proj_worker(void *arg)
{
    proj_job_t *J = (proj_job_t *)arg;
    float *a16 = malloc(sizeof(float) * (size_t)J->K);
    if (!a16) return NULL;
    for (;;) {
        const long t = atomic_fetch_add(&J->next, 1);
        if (t >= J->n) break;
        const float *a = J->A + t * J->lda;
        for (int k = 0; k < J->K; k++) a16[k] = J->mode == VTX_REF_FP64 ? a[k] : h2f(f2h(a[k]));
        for (int o = 0; o < J->N; o++) {
            const uint16_t *w = J->W + (int64_t)o * J->ldw;
            double y;
            if (J->mode == VTX_REF_FP64) {
                double s = 0.0;
                for (int k = 0; k < J->K; k++) s += (double)a16[k] * (double)h2f(w[k]);
                y = s;
            } else {
                float s = 0.0f;
                for (int k = 0; k < J->K; k++) s += a16[k] * h2f(w[k]);
                y = s;
            }
            if (J->mode == VTX_REF_FP64) {
                if (J->bias) y += J->bias[o];
                if (J->res) y += J->res[t * J->ldr + o];
                J->dst[t * J->ldd + o] = (float)y;
            } else {
                float yf = (float)y;
                if (J->bias) yf += J->bias[o];
                if (J->res) yf = J->res[t * J->ldr + o] + yf;
                J->dst[t * J->ldd + o] = yf;
            }
        }
    }
    free(a16);
    return NULL;
}

int vtx_ref_out_proj(const float *A, int64_t lda, const uint16_t *W, int64_t ldw, const float *bias,
                     const float *res, int64_t ldr, float *dst, int64_t ldd, int n, int K, int N, int mode,
                     int n_threads)
{
    if (!A || !W || !dst || n < 0 || K <= 0 || N <= 0) return VTX_ERR_SHAPE;
    proj_job_t J = {A, lda, W, ldw, bias, res, ldr, dst, ldd, n, K, N, mode, 0};
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (n < n_threads) n_threads = n > 0 ? n : 1;
    pthread_t th[256];
    for (int t = 1; t < n_threads; t++) pthread_create(&th[t], NULL, proj_worker, &J);
    proj_worker(&J);
    for (int t = 1; t < n_threads; t++) pthread_join(th[t], NULL);
    return 0;
}
