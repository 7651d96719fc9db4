/*
 * oracle/attn_ref.c — TEST INFRASTRUCTURE ONLY. CPU restatement (plain C, fp32, OpenMP) of hayatree/oumu's
 * attention hot path, used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker
 * and the CPU baseline. Nothing in the product (oumu_b200/) links, loads or calls it.
 *
 * Every function restates one reference kernel; citations are paths inside the reference repository.
 * Storage is bf16 (uint16_t bit patterns), arithmetic fp32, rounding to bf16 where the reference rounds.
 * Pinned against golden vectors produced by the reference kernels themselves (tests/golden/).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* bf16 round-to-nearest-even with NaN -> 0x7fc0: f2b of src/gpu.rs:72-78. */
uint16_t oracle_f2b(float x) {
    if (isnan(x)) return 0x7fc0;
    uint32_t u;
    memcpy(&u, &x, 4);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

/* b2f of src/gpu.rs:80-82. */
float oracle_b2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static float rb(float x) { return oracle_b2f(oracle_f2b(x)); }

int oracle_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/*
 * Rotary tables [maxlen][hd/2] (src/model.rs:337-349): inv = 1 / 10000^(2i/hd), fr = (p * (1/ext[i])) * inv,
 * cos/sin rounded through bf16. ext == NULL means 1 (plain base-10000 RoPE).
 */
void oracle_rotary_tables(int maxlen, int hd, const double *ext, float *cs, float *sn) {
    int half = hd / 2;
    for (int p = 0; p < maxlen; p++)
        for (int i = 0; i < half; i++) {
            float inv = 1.0f / powf(10000.0f, (float)(2 * i) / (float)hd);
            float e = ext ? (float)ext[i] : 1.0f;
            float fr = ((float)p * (1.0f / e)) * inv;
            cs[(long)p * half + i] = rb(cosf(fr));
            sn[(long)p * half + i] = rb(sinf(fr));
        }
}

/*
 * rope (kernels/voxcpm.cu:100-115), in place on the q and k heads of each row; position r % seq (seq > 0) or
 * *pos. x1' = bf16(x1*c - x2*s), x2' = bf16(x2*c + x1*s); the products are contracted into one fused
 * multiply-add the way CUDA compiles these two expressions (fma(x1, c, -(x2*s)), fma(x2, c, x1*s)).
 */
void oracle_rope(uint16_t *qkv, const float *cos_t, const float *sin_t, const int *pos, int rows, int seq, int nq,
                 int nk, int hd) {
    int half = hd / 2;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        int p = seq > 0 ? r % seq : *pos;
        for (int h = 0; h < nq + nk; h++) {
            uint16_t *v = qkv + (long)r * (nq + 2 * nk) * hd + (long)h * hd;
            for (int i = 0; i < half; i++) {
                float c = cos_t[(long)p * half + i], s = sin_t[(long)p * half + i];
                float x1 = oracle_b2f(v[i]), x2 = oracle_b2f(v[i + half]);
                v[i] = oracle_f2b(fmaf(x1, c, -(x2 * s)));
                v[i + half] = oracle_f2b(fmaf(x2, c, x1 * s));
            }
        }
    }
}

/*
 * kv_write (kernels/voxcpm.cu:117-129): k and v of rows i < rows of every slot s into
 * cache[((s*nk + h)*maxlen + p)*hd + d], p = (*pos or 0) + i; qkv row s*rows + i.
 */
void oracle_kv_write(const uint16_t *qkv, uint16_t *kc, uint16_t *vc, const int *pos, int slots, int rows, int nq,
                     int nk, int hd, int maxlen) {
    for (int s = 0; s < slots; s++)
        for (int i = 0; i < rows; i++)
            for (int h = 0; h < nk; h++) {
                int p = (pos ? *pos : 0) + i;
                const uint16_t *src = qkv + ((long)s * rows + i) * (nq + 2 * nk) * hd;
                long dst = (((long)s * nk + h) * maxlen + p) * hd;
                memcpy(kc + dst, src + (long)(nq + h) * hd, (size_t)hd * 2);
                memcpy(vc + dst, src + (long)(nq + nk + h) * hd, (size_t)hd * 2);
            }
}

/* kv_replicate (kernels/voxcpm.cu:407-413): slot 0 -> slots 1..B-1 for positions < T. */
void oracle_kv_replicate(uint16_t *c, int B, int nk, int maxlen, int hd, int T) {
    for (int s = 1; s < B; s++)
        for (int h = 0; h < nk; h++)
            for (int p = 0; p < T; p++)
                memcpy(c + (((long)s * nk + h) * maxlen + p) * hd, c + ((long)h * maxlen + p) * hd, (size_t)hd * 2);
}

#define ATT_CH 64 /* kernels/voxcpm.cu:134 */

/*
 * attn_decode + attn_combine (kernels/voxcpm.cu:131-185). For take s, q head h (kv head h / (nq/nk)):
 * per 64-position split sp < ceil(L/64) a partial (m, sum, acc[d]) with score = (q.k)*scale and e = exp(score-m),
 * then the log-sum-exp merge out = bf16(sum_i w_i acc_i / sum_i w_i sum_i), w_i = exp(m_i - max m).
 * L = lens[s] when lens != NULL (per-take lengths), else *pos + 1 for every take (the reference's shared position).
 * out is [B][nq*hd] bf16.
 */
void oracle_attn_decode(const uint16_t *qkv, const uint16_t *kc, const uint16_t *vc, uint16_t *out, const int *pos,
                        const int *lens, int B, int nq, int nk, int hd, int maxlen, float scale) {
    int grp = nq / nk;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int s = 0; s < B; s++)
        for (int h = 0; h < nq; h++) {
            int L = lens ? lens[s] : *pos + 1;
            int kh = h / grp;
            int nsp = (L + ATT_CH - 1) / ATT_CH;
            float q[256], acc_all[256], sc[ATT_CH];
            float *pm = (float *)malloc(sizeof(float) * (size_t)nsp * (hd + 2));
            const uint16_t *qr = qkv + (long)s * (nq + 2 * nk) * hd + (long)h * hd;
            for (int d = 0; d < hd; d++) q[d] = oracle_b2f(qr[d]);
            for (int sp = 0; sp < nsp; sp++) {
                int j0 = sp * ATT_CH, n = L - j0 < ATT_CH ? L - j0 : ATT_CH;
                const uint16_t *K = kc + (((long)s * nk + kh) * maxlen + j0) * hd;
                const uint16_t *V = vc + (((long)s * nk + kh) * maxlen + j0) * hd;
                float m = -INFINITY;
                for (int j = 0; j < n; j++) {
                    float a = 0.f;
                    for (int d = 0; d < hd; d++) a += q[d] * oracle_b2f(K[(long)j * hd + d]);
                    sc[j] = a * scale;
                    m = fmaxf(m, sc[j]);
                }
                float sum = 0.f;
                float *pr = pm + (long)sp * (hd + 2);
                for (int d = 0; d < hd; d++) pr[2 + d] = 0.f;
                for (int j = 0; j < n; j++) {
                    float e = expf(sc[j] - m);
                    sum += e;
                    for (int d = 0; d < hd; d++) pr[2 + d] += e * oracle_b2f(V[(long)j * hd + d]);
                }
                pr[0] = m;
                pr[1] = sum;
            }
            float M = -INFINITY;
            for (int i = 0; i < nsp; i++) M = fmaxf(M, pm[(long)i * (hd + 2)]);
            float tot = 0.f;
            for (int d = 0; d < hd; d++) acc_all[d] = 0.f;
            for (int i = 0; i < nsp; i++) {
                float *pr = pm + (long)i * (hd + 2);
                float w = expf(pr[0] - M);
                tot += w * pr[1];
                for (int d = 0; d < hd; d++) acc_all[d] += w * pr[2 + d];
            }
            uint16_t *o = out + (long)s * nq * hd + (long)h * hd;
            for (int d = 0; d < hd; d++) o[d] = oracle_f2b(acc_all[d] / tot);
            free(pm);
        }
}

/*
 * attn_full (kernels/voxcpm.cu:262-297): for query row r of sequence s0 = r - r%seq, keys j < (causal ? i+1 : seq)
 * with i = r % seq: sc[j] = (q.k_j)*scale, m = max, e_j = exp(sc[j] - m), inv = 1/sum e_j,
 * out = bf16((sum_j e_j v_j) * inv). out is [rows][nq*hd].
 */
void oracle_attn_full(const uint16_t *qkv, uint16_t *out, int rows, int seq, int causal, int nq, int nk, int hd,
                      float scale) {
    int grp = nq / nk, stride = (nq + 2 * nk) * hd;
#pragma omp parallel
    {
        float *sc = (float *)malloc(sizeof(float) * (size_t)seq);
        float q[256], a[256];
#pragma omp for collapse(2) schedule(dynamic, 16)
        for (int r = 0; r < rows; r++)
            for (int h = 0; h < nq; h++) {
                int kh = h / grp, s0 = r - r % seq, i = r % seq;
                int L = causal ? i + 1 : seq;
                for (int d = 0; d < hd; d++) q[d] = oracle_b2f(qkv[(long)r * stride + (long)h * hd + d]);
                float m = -INFINITY;
                for (int j = 0; j < L; j++) {
                    const uint16_t *k = qkv + (long)(s0 + j) * stride + (long)(nq + kh) * hd;
                    float acc = 0.f;
                    for (int d = 0; d < hd; d++) acc += q[d] * oracle_b2f(k[d]);
                    sc[j] = acc * scale;
                    m = fmaxf(m, sc[j]);
                }
                float sum = 0.f;
                for (int j = 0; j < L; j++) {
                    sc[j] = expf(sc[j] - m);
                    sum += sc[j];
                }
                float inv = 1.f / sum;
                for (int d = 0; d < hd; d++) a[d] = 0.f;
                for (int j = 0; j < L; j++) {
                    const uint16_t *v = qkv + (long)(s0 + j) * stride + (long)(nq + nk + kh) * hd;
                    for (int d = 0; d < hd; d++) a[d] += sc[j] * oracle_b2f(v[d]);
                }
                uint16_t *o = out + (long)r * nq * hd + (long)h * hd;
                for (int d = 0; d < hd; d++) o[d] = oracle_f2b(a[d] * inv);
            }
        free(sc);
    }
}
