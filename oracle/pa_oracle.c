/* pa_oracle.c - CPU restatement of phone-attn's partial attention (see pa_oracle.h for the map to the
 * reference). TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU baseline. */
#include "pa_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- binary16 */

uint16_t orc_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t) (sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u | ((ax >> 13) & 0x3ffu) : 0u));
    if (ax >= 0x477ff000u) return (uint16_t) (sign | 0x7c00u); /* >= 65520: rounds to inf */
    if (ax < 0x38800000u) {                                     /* result is subnormal (or zero) */
        if (ax <= 0x33000000u) return (uint16_t) sign;          /* <= 2^-25 rounds to zero (tie goes to even 0) */
        const uint32_t e = ax >> 23, mant = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e; /* value / 2^-24 = mant * 2^(e-126) */
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t) (sign | h);
    }
    uint32_t h = ((ax >> 23) - 112u) << 10 | ((ax >> 13) & 0x3ffu);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t) (sign | h);
}

float orc_h2f(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, mant = h & 0x3ffu, x;
    if (e == 0x1fu) {
        x = sign | 0x7f800000u | (mant << 13);
    } else if (e == 0) {
        if (mant == 0) {
            x = sign;
        } else { /* subnormal: normalise */
            e = 113;
            while (!(mant & 0x400u)) { mant <<= 1; e--; }
            x = sign | (e << 23) | ((mant & 0x3ffu) << 13);
        }
    } else {
        x = sign | ((e + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void orc_f2h_n(const float *x, uint16_t *h, size_t n) { for (size_t i = 0; i < n; i++) h[i] = orc_f2h(x[i]); }
void orc_h2f_n(const uint16_t *h, float *x, size_t n) { for (size_t i = 0; i < n; i++) x[i] = orc_h2f(h[i]); }

/* round a float to the nearest binary16 value (kept as float); the hot loops of the fp32 path use the
 * compiler's _Float16 (F16C instructions, also round to nearest even), the tests check both agree */
static inline float r16(float x) {
#if defined(__FLT16_MAX__)
    return (float) (_Float16) x;
#else
    return orc_h2f(orc_f2h(x));
#endif
}
static inline float h2f_fast(uint16_t h) {
#if defined(__FLT16_MAX__)
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float) v;
#else
    return orc_h2f(h);
#endif
}

/* ---------------------------------------------------------------- pa-tool's test rows */

float orc_lcg_frand(uint64_t *s) {
    *s = *s * 6364136223846793005ull + 1442695040888963407ull;
    return ((float) (*s >> 40) / (float) (1 << 24)) * 2 - 1;
}

void orc_pt_make_q8_row(uint8_t *row, int nkv, float amp, uint64_t *s) {
    for (int h = 0; h < nkv; h++)
        for (int b = 0; b < 8; b++) {
            float x[32], am = 0;
            for (int i = 0; i < 32; i++) { x[i] = orc_lcg_frand(s) * amp; am = fmaxf(am, fabsf(x[i])); }
            const float d = am / 127;
            const uint16_t dh = orc_f2h(d);
            uint8_t *o = row + h * 272 + b * 34;
            memcpy(o, &dh, 2);
            const float id = d != 0 ? 1 / orc_h2f(dh) : 0;
            for (int i = 0; i < 32; i++) o[2 + i] = (uint8_t) (int8_t) lrintf(fmaxf(-127.f, fminf(127.f, x[i] * id)));
        }
}

void orc_pt_make_q4_row(uint8_t *row, int nkv, float amp, uint64_t *s) {
    for (int h = 0; h < nkv; h++)
        for (int b = 0; b < 8; b++) {
            float x[32], am = 0, mx = 0;
            for (int i = 0; i < 32; i++) {
                x[i] = orc_lcg_frand(s) * amp;
                if (fabsf(x[i]) > am) { am = fabsf(x[i]); mx = x[i]; }
            }
            const float d = mx / -8;
            const uint16_t dh = orc_f2h(d);
            uint8_t *o = row + h * 144 + b * 18;
            memcpy(o, &dh, 2);
            const float id = d != 0 ? 1 / orc_h2f(dh) : 0;
            for (int i = 0; i < 16; i++) {
                int lo = (int) (x[i] * id + 8.5f), hi = (int) (x[i + 16] * id + 8.5f);
                lo = lo < 15 ? lo : 15; hi = hi < 15 ? hi : 15;
                lo = lo > 0 ? lo : 0;   hi = hi > 0 ? hi : 0;
                o[2 + i] = (uint8_t) (lo | (hi << 4));
            }
        }
}

/* ---------------------------------------------------------------- formats */

size_t orc_head_bytes(int quant, int hd) {
    return quant == ORC_Q8_0 ? (size_t) hd / 32 * 34 : quant == ORC_Q4_0 ? (size_t) hd / 32 * 18 : (size_t) hd * 2;
}

float orc_deq(const uint8_t *row, int quant, int hd, int h, int d) {
    const size_t hb = orc_head_bytes(quant, hd);
    const uint8_t *hp = row + (size_t) h * hb;
    if (quant == ORC_F16) {
        uint16_t v;
        memcpy(&v, hp + 2 * d, 2);
        return orc_h2f(v);
    }
    if (quant == ORC_Q4_0) {
        const uint8_t *blk = hp + (d / 32) * 18;
        uint16_t dh;
        memcpy(&dh, blk, 2);
        const int i = d % 32;
        const uint8_t q = blk[2 + (i % 16)];
        return orc_h2f(dh) * (float) ((i < 16 ? (q & 15) : (q >> 4)) - 8);
    }
    const uint8_t *blk = hp + (d / 32) * 34;
    uint16_t dh;
    memcpy(&dh, blk, 2);
    return orc_h2f(dh) * (float) (int8_t) blk[2 + d % 32];
}

void orc_quant_q8_0(const float *x, size_t n_blocks, uint8_t *out) {
    for (size_t b = 0; b < n_blocks; b++) {
        const float *xb = x + b * 32;
        float am = 0;
        for (int i = 0; i < 32; i++) am = fmaxf(am, fabsf(xb[i]));
        const uint16_t dh = orc_f2h(am / 127);
        uint8_t *o = out + b * 34;
        memcpy(o, &dh, 2);
        const float df = orc_h2f(dh), id = df != 0 ? 1 / df : 0;
        for (int i = 0; i < 32; i++) o[2 + i] = (uint8_t) (int8_t) lrintf(fmaxf(-127.f, fminf(127.f, xb[i] * id)));
    }
}

void orc_quant_q4_0(const float *x, size_t n_blocks, uint8_t *out) {
    for (size_t b = 0; b < n_blocks; b++) {
        const float *xb = x + b * 32;
        float am = 0;
        for (int i = 0; i < 32; i++) am = fmaxf(am, fabsf(xb[i]));
        const uint16_t dh = orc_f2h(am / 7);
        uint8_t *o = out + b * 18;
        memcpy(o, &dh, 2);
        const float df = orc_h2f(dh), id = df != 0 ? 1 / df : 0;
        int q[32];
        for (int i = 0; i < 32; i++) {
            long v = lrintf(xb[i] * id) + 8;
            q[i] = (int) (v < 1 ? 1 : v > 15 ? 15 : v);
        }
        for (int i = 0; i < 16; i++) o[2 + i] = (uint8_t) (q[i] | (q[i + 16] << 4));
    }
}

void orc_scale_q(const float *Q, float scale, uint16_t *Qs, size_t n) {
    for (size_t i = 0; i < n; i++) Qs[i] = orc_f2h(Q[i] * scale);
}

/* ---------------------------------------------------------------- fp64 reference */

void orc_partial_f64(const orc_shape *sh, const uint16_t *Qs, const uint8_t *K, const uint8_t *V, uint32_t nk,
                     double *O, double *m, double *l) {
    const int hd = sh->hd;
    double *kf = (double *) malloc(sizeof(double) * (size_t) (nk ? nk : 1) * hd);
    double *vf = (double *) malloc(sizeof(double) * (size_t) (nk ? nk : 1) * hd);
    double *s = (double *) malloc(sizeof(double) * (nk ? nk : 1));
    double *q = (double *) malloc(sizeof(double) * hd);
    for (int h = 0; h < sh->nkv; h++) {
        for (uint32_t j = 0; j < nk; j++)
            for (int d = 0; d < hd; d++) {
                kf[(size_t) j * hd + d] = orc_deq(K + (size_t) j * sh->rs + (size_t) h * sh->hb, sh->quant, hd, 0, d);
                vf[(size_t) j * hd + d] = orc_deq(V + (size_t) j * sh->rs + (size_t) h * sh->hb, sh->quant, hd, 0, d);
            }
        for (int r = 0; r < sh->rows; r++) {
            const size_t row = (size_t) h * sh->rows + r;
            double *o = O + row * hd;
            for (int d = 0; d < hd; d++) { q[d] = orc_h2f(Qs[row * hd + d]); o[d] = 0; }
            if (nk == 0) { m[row] = -INFINITY; l[row] = 0; continue; }
            double mx = -INFINITY;
            for (uint32_t j = 0; j < nk; j++) {
                double a = 0;
                for (int d = 0; d < hd; d++) a += q[d] * kf[(size_t) j * hd + d];
                s[j] = a;
                if (a > mx) mx = a;
            }
            double L = 0;
            for (uint32_t j = 0; j < nk; j++) {
                const double p = exp(s[j] - mx);
                L += p;
                for (int d = 0; d < hd; d++) o[d] += p * vf[(size_t) j * hd + d];
            }
            m[row] = mx;
            l[row] = L;
        }
    }
    free(kf); free(vf); free(s); free(q);
}

/* ---------------------------------------------------------------- fp32 block online softmax */

/* dequantise keys [0, b) of head h to f16-rounded floats: transposed dT[d][b] (K) or row-major d[j][hd] (V) */
static void deq_block(const orc_shape *sh, const uint8_t *X, int b, int h, float *dst, int transposed, int ld) {
    const int hd = sh->hd;
    for (int j = 0; j < b; j++) {
        const uint8_t *hp = X + (size_t) j * sh->rs + (size_t) h * sh->hb;
        for (int blk = 0; blk < hd / 32; blk++) {
            float v[32];
            if (sh->quant == ORC_Q8_0) {
                const uint8_t *p = hp + blk * 34;
                uint16_t dh;
                memcpy(&dh, p, 2);
                const float dd = h2f_fast(dh);
                for (int i = 0; i < 32; i++) v[i] = r16(dd * (float) (int8_t) p[2 + i]);
            } else if (sh->quant == ORC_Q4_0) {
                const uint8_t *p = hp + blk * 18;
                uint16_t dh;
                memcpy(&dh, p, 2);
                const float dd = h2f_fast(dh);
                for (int i = 0; i < 16; i++) {
                    v[i] = r16(dd * (float) ((p[2 + i] & 15) - 8));
                    v[i + 16] = r16(dd * (float) ((p[2 + i] >> 4) - 8));
                }
            } else {
                for (int i = 0; i < 32; i++) {
                    uint16_t x;
                    memcpy(&x, hp + 2 * (blk * 32 + i), 2);
                    v[i] = h2f_fast(x);
                }
            }
            for (int i = 0; i < 32; i++) {
                const int d = blk * 32 + i;
                if (transposed) dst[(size_t) d * ld + j] = v[i];
                else dst[(size_t) j * ld + d] = v[i];
            }
        }
    }
}

void orc_partial_f32(const orc_shape *sh, const uint16_t *Qs, const uint8_t *K, const uint8_t *V, uint32_t nk,
                     int bk, int h0, int h1, float *O, float *m, float *l) {
    const int hd = sh->hd, R = sh->rows;
    if (bk <= 0) bk = 512;
    float *kT = (float *) malloc(sizeof(float) * (size_t) hd * bk);
    float *vb = (float *) malloc(sizeof(float) * (size_t) bk * hd);
    float *S = (float *) malloc(sizeof(float) * (size_t) R * bk);
    float *q = (float *) malloc(sizeof(float) * (size_t) R * hd);
    float *Ot = (float *) malloc(sizeof(float) * (size_t) R * hd);
    float *alpha = (float *) malloc(sizeof(float) * R);
    for (int h = h0; h < h1; h++) {
        float *Oh = O + (size_t) h * R * hd, *mh = m + (size_t) h * R, *lh = l + (size_t) h * R;
        for (int i = 0; i < R * hd; i++) q[i] = h2f_fast(Qs[(size_t) h * R * hd + i]);
        for (int r = 0; r < R; r++) { mh[r] = -1e30f; lh[r] = 0; }
        memset(Oh, 0, sizeof(float) * (size_t) R * hd);
        for (uint32_t j0 = 0; j0 < nk; j0 += (uint32_t) bk) {
            const int b = nk - j0 < (uint32_t) bk ? (int) (nk - j0) : bk;
            deq_block(sh, K + (size_t) j0 * sh->rs, b, h, kT, 1, bk);
            for (int r = 0; r < R; r++) {
                float *sr = S + (size_t) r * bk;
                for (int j = 0; j < b; j++) sr[j] = 0;
                for (int d = 0; d < hd; d++) {
                    const float qv = q[(size_t) r * hd + d];
                    const float *kd = kT + (size_t) d * bk;
                    for (int j = 0; j < b; j++) sr[j] += qv * kd[j];
                }
            }
            /* softmax_blk (sme_attn.c:216-243): P rounded to f16, l += sum of the fp32 p */
            for (int r = 0; r < R; r++) {
                float *sr = S + (size_t) r * bk;
                float mx = -INFINITY;
                for (int j = 0; j < b; j++) mx = fmaxf(mx, sr[j]);
                const float mn = fmaxf(mh[r], mx);
                alpha[r] = expf(mh[r] - mn);
                mh[r] = mn;
                float ls = 0;
                for (int j = 0; j < b; j++) {
                    const float p = expf(sr[j] - mn);
                    ls += p;
                    sr[j] = r16(p);
                }
                lh[r] = fmaf(lh[r], alpha[r], ls);
            }
            deq_block(sh, V + (size_t) j0 * sh->rs, b, h, vb, 0, hd);
            for (int r = 0; r < R; r++) {
                float *ot = Ot + (size_t) r * hd;
                const float *pr = S + (size_t) r * bk;
                for (int d = 0; d < hd; d++) ot[d] = 0;
                for (int j = 0; j < b; j++) {
                    const float p = pr[j];
                    const float *vj = vb + (size_t) j * hd;
                    for (int d = 0; d < hd; d++) ot[d] += p * vj[d];
                }
                float *o = Oh + (size_t) r * hd;
                for (int d = 0; d < hd; d++) o[d] = fmaf(o[d], alpha[r], ot[d]);
            }
        }
    }
    free(kT); free(vb); free(S); free(q); free(Ot); free(alpha);
}

/* The int8-domain QK of scripts/sme/sme_attn.c:465-508 (sme_qk_i8blk: per 32-block int32 dot products of int8 Q and
 * q8_0 K; i8_combine: s = sum_b float(T_b) * (dq_b * dk_b)), with Q quantised per 32-block by the Q8_0 rule
 * (orc_quant_q8_0: d = f16(max|x|/127), q = rint(x / d); the reference leaves Q's rule to its caller), applied to the
 * f16(q*scale) values the kernels receive. Softmax and P.V as orc_partial_f32 (P and V rounded to f16). Q8_0 rows only;
 * returns -1 for other formats. */
int orc_partial_f32_i8q(const orc_shape *sh, const uint16_t *Qs, const uint8_t *K, const uint8_t *V, uint32_t nk,
                        int bk, int h0, int h1, float *O, float *m, float *l) {
    if (sh->quant != ORC_Q8_0) return -1;
    const int hd = sh->hd, R = sh->rows, NB = hd / 32;
    if (bk <= 0) bk = 512;
    int8_t *qi = (int8_t *) malloc((size_t) R * hd);
    float *dq = (float *) malloc(sizeof(float) * (size_t) R * NB);
    float *vb = (float *) malloc(sizeof(float) * (size_t) bk * hd);
    float *S = (float *) malloc(sizeof(float) * (size_t) R * bk);
    float *Ot = (float *) malloc(sizeof(float) * (size_t) R * hd);
    float *alpha = (float *) malloc(sizeof(float) * R);
    uint8_t blk[34];
    for (int h = h0; h < h1; h++) {
        float *Oh = O + (size_t) h * R * hd, *mh = m + (size_t) h * R, *lh = l + (size_t) h * R;
        for (int r = 0; r < R; r++)
            for (int b = 0; b < NB; b++) {
                float x[32];
                for (int i = 0; i < 32; i++) x[i] = h2f_fast(Qs[((size_t) h * R + r) * hd + b * 32 + i]);
                orc_quant_q8_0(x, 1, blk);
                uint16_t dh;
                memcpy(&dh, blk, 2);
                dq[(size_t) r * NB + b] = h2f_fast(dh);
                for (int i = 0; i < 32; i++) qi[((size_t) r * NB + b) * 32 + i] = (int8_t) blk[2 + i];
            }
        for (int r = 0; r < R; r++) { mh[r] = -1e30f; lh[r] = 0; }
        memset(Oh, 0, sizeof(float) * (size_t) R * hd);
        for (uint32_t j0 = 0; j0 < nk; j0 += (uint32_t) bk) {
            const int b = nk - j0 < (uint32_t) bk ? (int) (nk - j0) : bk;
            for (int j = 0; j < b; j++) {
                const uint8_t *hp = K + (size_t) (j0 + j) * sh->rs + (size_t) h * sh->hb;
                for (int r = 0; r < R; r++) {
                    float acc = 0;
                    for (int q = 0; q < NB; q++) {
                        const uint8_t *p = hp + q * 34;
                        uint16_t dh;
                        memcpy(&dh, p, 2);
                        int32_t t = 0;
                        const int8_t *qr = qi + ((size_t) r * NB + q) * 32;
                        for (int i = 0; i < 32; i++) t += (int32_t) qr[i] * (int32_t) (int8_t) p[2 + i];
                        acc = fmaf((float) t, dq[(size_t) r * NB + q] * h2f_fast(dh), acc);
                    }
                    S[(size_t) r * bk + j] = acc;
                }
            }
            for (int r = 0; r < R; r++) {
                float *sr = S + (size_t) r * bk;
                float mx = -INFINITY;
                for (int j = 0; j < b; j++) mx = fmaxf(mx, sr[j]);
                const float mn = fmaxf(mh[r], mx);
                alpha[r] = expf(mh[r] - mn);
                mh[r] = mn;
                float ls = 0;
                for (int j = 0; j < b; j++) {
                    const float p = expf(sr[j] - mn);
                    ls += p;
                    sr[j] = r16(p);
                }
                lh[r] = fmaf(lh[r], alpha[r], ls);
            }
            deq_block(sh, V + (size_t) j0 * sh->rs, b, h, vb, 0, hd);
            for (int r = 0; r < R; r++) {
                float *ot = Ot + (size_t) r * hd;
                const float *pr = S + (size_t) r * bk;
                for (int d = 0; d < hd; d++) ot[d] = 0;
                for (int j = 0; j < b; j++) {
                    const float p = pr[j];
                    const float *vj = vb + (size_t) j * hd;
                    for (int d = 0; d < hd; d++) ot[d] += p * vj[d];
                }
                float *o = Oh + (size_t) r * hd;
                for (int d = 0; d < hd; d++) o[d] = fmaf(o[d], alpha[r], ot[d]);
            }
        }
    }
    free(qi); free(dq); free(vb); free(S); free(Ot); free(alpha);
    return 0;
}

/* ---------------------------------------------------------------- merges */

void orc_merge_partial(float *O, float *m, float *l, const float *O2, const float *m2, const float *l2, size_t rows,
                       int hd) {
    for (size_t r = 0; r < rows; r++) {
        if (l2[r] <= 0) continue;
        if (l[r] <= 0) {
            memcpy(O + r * hd, O2 + r * hd, (size_t) hd * sizeof(float));
            m[r] = m2[r];
            l[r] = l2[r];
            continue;
        }
        const float M = fmaxf(m[r], m2[r]), a = expf(m[r] - M), b = expf(m2[r] - M);
        for (int d = 0; d < hd; d++) O[r * hd + d] = O[r * hd + d] * a + O2[r * hd + d] * b;
        m[r] = M;
        l[r] = l[r] * a + l2[r] * b;
    }
}

void orc_merge_slots(const float *Op, const float *mp, const float *lp, int n_slots, size_t rows, int hd, float *O,
                     float *m, float *l) {
    for (size_t r = 0; r < rows; r++) {
        float M = -INFINITY;
        for (int c = 0; c < n_slots; c++) M = fmaxf(M, mp[(size_t) c * rows + r]);
        float L = 0;
        float *o = O + r * hd;
        for (int d = 0; d < hd; d++) o[d] = 0;
        for (int c = 0; c < n_slots; c++) {
            const float mc = mp[(size_t) c * rows + r];
            if (mc == -INFINITY) continue;
            const float w = expf(mc - M);
            L += w * lp[(size_t) c * rows + r];
            const float *oc = Op + ((size_t) c * rows + r) * hd;
            for (int d = 0; d < hd; d++) o[d] += w * oc[d];
        }
        m[r] = M;
        l[r] = L;
    }
}

void orc_normalize(const float *O, const float *m, const float *l, size_t rows, int hd, uint16_t *Oh, float *lse) {
    for (size_t r = 0; r < rows; r++) {
        const float inv = l[r] > 0 ? 1.0f / l[r] : 0.0f;
        for (int d = 0; d < hd; d++) Oh[r * hd + d] = orc_f2h(O[r * hd + d] * inv);
        lse[r] = l[r] > 0 ? m[r] + logf(l[r]) : -INFINITY;
    }
}

/* ---------------------------------------------------------------- multi-threaded fp32 path */

typedef struct {
    const orc_shape *sh;
    const uint16_t *Qs;
    const uint8_t *K, *V;
    uint32_t nk, chunk;
    int n_chunks, n_items;
    float *Oi, *mi, *li; /* per item: [rows][hd], [rows], [rows] */
    atomic_int next;
} mt_job;

static void *mt_worker(void *arg) {
    mt_job *J = (mt_job *) arg;
    const orc_shape *sh = J->sh;
    const size_t rows = (size_t) sh->rows, hd = (size_t) sh->hd;
    for (;;) {
        const int it = atomic_fetch_add(&J->next, 1);
        if (it >= J->n_items) break;
        const int h = it / J->n_chunks, c = it % J->n_chunks;
        const uint32_t j0 = (uint32_t) c * J->chunk, n = J->nk - j0 < J->chunk ? J->nk - j0 : J->chunk;
        /* orc_partial_f32 writes head h at offset h*rows: shift the base (it >= h) so that head h lands on this
         * item's buffers */
        float *O = J->Oi + (size_t) (it - h) * rows * hd;
        float *m = J->mi + (size_t) (it - h) * rows;
        float *l = J->li + (size_t) (it - h) * rows;
        orc_partial_f32(sh, J->Qs, J->K + (size_t) j0 * sh->rs, J->V + (size_t) j0 * sh->rs, n, 512, h, h + 1, O, m, l);
    }
    return NULL;
}

int orc_partial_f32_mt(const orc_shape *sh, const uint16_t *Qs, const uint8_t *K, const uint8_t *V, uint32_t nk,
                       int nthreads, uint32_t chunk_keys, float *O, float *m, float *l) {
    const size_t rows = (size_t) sh->rows, hd = (size_t) sh->hd;
    if (chunk_keys == 0) chunk_keys = 4096;
    if (nthreads < 1) nthreads = 1;
    mt_job J;
    J.sh = sh; J.Qs = Qs; J.K = K; J.V = V; J.nk = nk; J.chunk = chunk_keys;
    J.n_chunks = nk ? (int) ((nk + chunk_keys - 1) / chunk_keys) : 0;
    J.n_items = J.n_chunks * sh->nkv;
    atomic_init(&J.next, 0);
    for (size_t i = 0; i < (size_t) sh->nkv * rows; i++) { m[i] = -INFINITY; l[i] = 0; }
    memset(O, 0, sizeof(float) * (size_t) sh->nkv * rows * hd);
    if (J.n_items == 0) return 0;
    J.Oi = (float *) malloc(sizeof(float) * (size_t) J.n_items * rows * hd);
    J.mi = (float *) malloc(sizeof(float) * (size_t) J.n_items * rows);
    J.li = (float *) malloc(sizeof(float) * (size_t) J.n_items * rows);
    if (!J.Oi || !J.mi || !J.li) { free(J.Oi); free(J.mi); free(J.li); return -1; }
    pthread_t *th = (pthread_t *) malloc(sizeof(pthread_t) * (size_t) nthreads);
    int *ok = (int *) calloc((size_t) nthreads, sizeof(int));
    for (int t = 1; t < nthreads; t++) ok[t] = pthread_create(&th[t], NULL, mt_worker, &J) == 0;
    mt_worker(&J);
    for (int t = 1; t < nthreads; t++) if (ok[t]) pthread_join(th[t], NULL);
    free(th);
    free(ok);
    for (int it = 0; it < J.n_items; it++) {
        const int h = it / J.n_chunks;
        orc_merge_partial(O + (size_t) h * rows * hd, m + (size_t) h * rows, l + (size_t) h * rows,
                          J.Oi + (size_t) it * rows * hd, J.mi + (size_t) it * rows, J.li + (size_t) it * rows, rows,
                          (int) hd);
    }
    free(J.Oi); free(J.mi); free(J.li);
    return 0;
}
