/* pa_oracle.h - CPU restatement of Backburner's phone-attn partial attention.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA path is compared against (and the
 * timed CPU baseline leg of bench.py). Nothing in the product library links or calls it.
 *
 * Every function restates a piece of the reference (paths relative to the reference repo):
 *   orc_f2h / orc_h2f            phone-attn/phone-attn.h:120-121 (IEEE binary16, round to nearest even)
 *   orc_lcg_frand                phone-attn/pa-tool.cpp:16-17, scripts/sme/sme_attn.c:561
 *   orc_pt_make_q8_row           phone-attn/pa-tool.cpp:20-27   (pa-tool's q8_0 test rows, HD 256)
 *   orc_pt_make_q4_row           phone-attn/pa-tool.cpp:29-40   (pa-tool's q4_0 test rows, ggml signed-max/-8)
 *   orc_deq                      phone-attn/pa-tool.cpp:41-51   (exact dequant, generalised to any head dim)
 *   orc_quant_q8_0               phone-attn/pa-tool.cpp:22-25   (d = max|x|/127 as f16, q = rint(x / f16(d)))
 *   orc_quant_q4_0               BASELINE Q4_0 rule: d = max|x|/7, q = rint(x/d) + 8 in [1,15], byte i = q[i] | q[i+16] << 4
 *   orc_partial_f64              phone-attn/pa-tool.cpp:150-173, scripts/sme/sme_attn.c:641-676 (fp64 reference)
 *   orc_partial_f32              scripts/sme/sme_attn.c:274-306 (block online softmax, f16 K/V/P, fp32 accumulators)
 *   orc_partial_f32_i8q          the same with the int8-domain QK of scripts/sme/sme_attn.c:465-508 (sme_qk_i8blk,
 *                                i8_combine), Q quantised per 32-block by the Q8_0 rule
 *   orc_partial_f32_mt           the same over (head x key chunk) threads, chunks folded with orc_merge_partial
 *   orc_merge_partial            phone-attn/phone-attn.h:231-239 (generalised to any head dim)
 *   orc_merge_slots              phone-attn/pa-metal.mm:137-159  (pa_merge: LSE fold of chunk slots)
 *   orc_normalize                phone-attn/phone-attn.h:651-655 (O/l -> f16, lse = m + log l)
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Quantisation of the held rows: the values of config_req.is_q8 (phone-attn/phone-attn.h:15). */
enum { ORC_F16 = 0, ORC_Q8_0 = 1, ORC_Q4_0 = 2 };

/* Geometry of one partial-attention call.
 *   hd    head dim (multiple of 32)
 *   nkv   KV heads
 *   rows  query rows per KV head (tokens x GQA group; the wire format uses 48 = 8 x 6)
 *   quant ORC_F16 / ORC_Q8_0 / ORC_Q4_0
 *   rs    bytes per key position (all heads); hb bytes per head inside a position
 * Q (f16 bits, already multiplied by the softmax scale) is [nkv][rows][hd]; K/V position j, head h
 * starts at K + j*rs + h*hb; O is [nkv][rows][hd], m and l are [nkv][rows]. */
typedef struct {
    int hd, nkv, rows, quant;
    size_t rs, hb;
} orc_shape;

size_t orc_head_bytes(int quant, int hd);

uint16_t orc_f2h(float f);
float    orc_h2f(uint16_t h);
void     orc_f2h_n(const float *x, uint16_t *h, size_t n);
void     orc_h2f_n(const uint16_t *h, float *x, size_t n);

float orc_lcg_frand(uint64_t *state);
void  orc_pt_make_q8_row(uint8_t *row, int nkv, float amp, uint64_t *state);
void  orc_pt_make_q4_row(uint8_t *row, int nkv, float amp, uint64_t *state);

float orc_deq(const uint8_t *row, int quant, int hd, int h, int d);
void  orc_quant_q8_0(const float *x, size_t n_blocks, uint8_t *out);
void  orc_quant_q4_0(const float *x, size_t n_blocks, uint8_t *out);

/* f16(q * scale) for n values of fp32 Q (scripts/sme/sme_attn.c:276-280) */
void orc_scale_q(const float *Q, float scale, uint16_t *Qs, size_t n);

/* fp64 reference partial over keys [0, nk): O = sum_j exp(s_j - m) v_j, l = sum_j exp(s_j - m),
 * m = max_j s_j, s_j = Qs . k_j, with exactly dequantised K/V. nk == 0 gives m = -inf, l = 0, O = 0. */
void orc_partial_f64(const orc_shape *sh, const uint16_t *Qs, const uint8_t *K, const uint8_t *V, uint32_t nk,
                     double *O, double *m, double *l);

/* fp32 block online softmax with bk-key blocks. K/V are dequantised to f16 (f16(d * q)), P is rounded to
 * f16 before P.V, m starts at -1e30 as in the reference. heads [h0, h1) only. */
void orc_partial_f32(const orc_shape *sh, const uint16_t *Qs, const uint8_t *K, const uint8_t *V, uint32_t nk,
                     int bk, int h0, int h1, float *O, float *m, float *l);

/* The same with the int8-domain QK of scripts/sme/sme_attn.c:465-508: Q quantised per 32-block (Q8_0 rule), per-block
 * int32 dot products with the q8_0 K integers, s = sum_b float(T_b) * (dq_b * dk_b). Q8_0 rows only (else -1). */
int orc_partial_f32_i8q(const orc_shape *sh, const uint16_t *Qs, const uint8_t *K, const uint8_t *V, uint32_t nk,
                        int bk, int h0, int h1, float *O, float *m, float *l);

/* orc_partial_f32 on nthreads pthreads over (head, chunk of chunk_keys) items; chunk partials of a head are
 * folded in key order. Returns 0 on success. */
int orc_partial_f32_mt(const orc_shape *sh, const uint16_t *Qs, const uint8_t *K, const uint8_t *V, uint32_t nk,
                       int nthreads, uint32_t chunk_keys, float *O, float *m, float *l);

void orc_merge_partial(float *O, float *m, float *l, const float *O2, const float *m2, const float *l2, size_t rows,
                       int hd);
/* fold n_slots partials laid out [slot][rows][hd] / [slot][rows] into one (pa_merge semantics) */
void orc_merge_slots(const float *Op, const float *mp, const float *lp, int n_slots, size_t rows, int hd, float *O,
                     float *m, float *l);
void orc_normalize(const float *O, const float *m, const float *l, size_t rows, int hd, uint16_t *Oh, float *lse);

#ifdef __cplusplus
}
#endif
