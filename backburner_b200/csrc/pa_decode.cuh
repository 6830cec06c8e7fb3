// pa_decode.cuh - split-K partial attention over quantised (Q8_0 / Q4_0) key/value rows, for the query shapes of
// decode and verify calls (a few rows per KV head).
//
// Reference semantics: pa_attn_big (phone-attn/pa-metal.mm:379-487) and sme_attn_partial
// (scripts/sme/sme_attn.c:274-306): K/V blocks are dequantised to f16 (f16(d * q)), S = Qs.K^T with fp32
// accumulation, online softmax in fp32 with P rounded to f16, O = diag(alpha) O + P.V, tail keys masked
// (pa-metal.mm:452-464). Output per chunk of keys: the unnormalised partial (O, m, l); pa_merge.cuh folds chunks.
//
// B200 design (one CTA = one key chunk x a group of heads x a group of query rows):
//   * each stage of K and V rows (16 keys) is streamed from HBM into shared memory with 1-D
//     bulk copies (TMA engine), one copy per PAIR of key rows (requests of one 1 KB row cap a B200 at ~5.4 TB/s, two
//     rows reach ~7.4 TB/s), pairs padded to an odd number of 16-byte units; NSTAGE stages ring on "full" mbarriers;
//     the last warp to finish with a stage (a shared counter) refills it, so there is no producer warp and every warp
//     of the CTA computes. At hd 128 a CTA has 8 warps of 128 registers and two CTAs share an SM: their stage rings
//     run independently (one 16-warp CTA with 32-key stages measured 6% slower);
//   * the MMA's 16 key rows are ordered even keys first (row g = key 2g, row g+8 = key 2g+1): with the pair layout
//     every 32-bit shared-memory read of K and V hits at most 2 lanes per bank;
//   * each consumer warp owns one (head, 8-row group) and, when there are few such groups, every other 16-key tile;
//   * the raw int8/int4 bytes go straight from shared memory into registers and are dequantised there into the
//     operand fragments of mma.m16n8k16 (f16 in, fp32 accumulate), keys on the M side ("swap AB"):
//       S^T[16 keys][8 rows] = K[16 keys][d] . Qs^T,   O^T[d][8 rows] += V^T[d][16 keys] . P^T
//     Because QK^T sums over d, the order of d inside a k-step is free: each lane takes whole 4-byte groups of its
//     own quant block (Q's fragments use the same permutation), so one scale per lane and no unpacking shuffles.
//     V needs keys in pairs along k: two rows' words are byte-interleaved with one PRMT. P's accumulator fragment
//     becomes P^T's operand fragment with movmatrix (8x8 transpose).
//   * P is taken against a lazily raised reference max (one warp vote per tile; the cross-lane max and the O rescale
//     run only when a score passes the reference by 2^8), and the exact row max is restored once per job; a tile's V
//     words are loaded before its softmax so their shared-memory latency overlaps the softmax.
//   * QUANT 3: Q8_0 rows with the int8-domain QK of scripts/sme/sme_attn.c:465-508 (sme_qk_i8blk + i8_combine): Q is
//     quantised per 32-block by the Q8_0 rule (d = f16(max|x| / 127), q = rint(x / d)) when a job starts, one
//     mma.m16n8k32 s8 per quant block gives the block's exact int32 dot products T for 16 keys x 8 rows, and
//     s = sum_b float(T_b) * (dq_b * dk_b) in block order (fma). Softmax and P.V are those of QUANT 1.
#pragma once
#include "pa_common.cuh"

namespace pa {
namespace dec {

// keys per pipeline stage: one 16-key MMA tile, so the tile loop of a stage is a compile-time single iteration; one lane
// copies a pair of rows
__host__ __device__ constexpr int stage_keys(int hd) { return 16; }
// stages in a CTA's ring: 3 at hd 128; 2 at hd 256, whose rows are twice as long
__host__ __device__ constexpr int nstage(int hd) { return hd == 128 ? 3 : 2; }
// Warps per CTA (W, the kernel's third parameter) and CTAs per SM for the register budget: hd 128: 8-warp CTAs, two
// per SM (two independent stage rings); hd 256: 8-warp CTAs, one per SM, with the ~206 registers a thread the O and Q
// fragments of 256 dims want (8 KV heads per CTA), or 4-warp CTAs, three per SM within 170 registers (fewer heads).
// Measured at hd 256, 16 layers x 64-131k Q8_0 keys: 8 heads x 6 rows 5,381 GB/s (8-warp) vs 4,920 (4-warp) and
// 2,835 with 32-key stages in 12-warp CTAs; 4 heads x 8 rows 5,521 (4-warp) vs 4,986 (8-warp).
__host__ __device__ constexpr int min_ctas(int hd, int w) { return hd == 128 ? 2 : (w == 4 ? 3 : 1); }
constexpr int TILE_KEYS = 16;    // keys per MMA tile
constexpr int SMEM_SLACK = 64;   // readable bytes past the last row (a lane may load one unused word there)
constexpr uint64_t DRAIN_NS = 1000000000ull;   // bound on waiting for copies in flight after an abort (>= 1 s)

// one chunk of keys of one segment, and where its partial goes
struct Job {
    const uint8_t *k, *v;   // segment base (key 0 of the segment)
    uint32_t key0, nk;      // keys [key0, key0 + nk) of the segment
    uint32_t set, slot;     // output set (selects Q) and partial slot
    uint32_t seg, pad_;     // segment index (selects the tensor maps of the tcgen05 kernel)
};

struct Params {
    const Job *jobs;
    const uint16_t *Qs;   // f16(q*scale) [n_sets][nkv][rows][hd]
    float *Op;            // partials [slot][nkv][rows][hd]
    float *Mp, *Lp;       // [slot][nkv][rows]
    int *status;
    uint64_t rs, hb;      // bytes per key position; bytes per head in a position
    uint32_t nkv, rows;
    uint32_t hg;          // heads per CTA
    uint32_t rgc;         // 8-row groups per CTA
    uint32_t n_rg;        // 8-row groups in total = ceil(rows / 8)
    uint32_t row;         // bytes of one key row in shared memory (= hg * hb, a multiple of 16)
    uint32_t gs;          // shared-memory stride of a pair of key rows (multiple of 16, odd number of 16-byte units)
    uint32_t n_jobs;      // jobs of the launch: CTA x takes jobs x, x + gridDim.x, ...
    uint32_t n_consumers; // warps per CTA (launch shape)
    uint64_t timeout_ns;
    int stall;            // test hook: consumers first wait on a barrier that nothing completes (bounded)
};

__host__ __device__ constexpr int q_group_bytes(int quant) { return quant == 1 ? 34 : quant == 2 ? 18 : 64; }

// ---------------------------------------------------------------- d permutations (host + device)
// QK^T: lane t of a quad feeds k = {2t, 2t+1, 2t+8, 2t+9} of each k-step s. Those 4 values are one 4-byte group of the
// lane's own quant block. dK(s, t, i) is the head-dim index of the i-th of them (i: 0,1 -> k = 2t,2t+1; 2,3 -> 2t+8,2t+9).
__host__ __device__ inline int dK(int quant, int s, int t, int i) {
    // f16 rows: natural order (ldmatrix fragments): k = 2t, 2t+1 -> d 16s + 2t + i; k = 2t+8, 2t+9 -> d 16s + 8 + 2t + i-2
    if (quant == 0) return 16 * s + 2 * t + (i < 2 ? i : 6 + i);
    const int blk = t + 4 * (s / 8), ss = s % 8;
    if (quant == 1) {
        // a pair of q8_0 blocks = 68 bytes = 17 aligned words; even block: (d,q0,q1)(q2..q5)...(q30,q31,d'), odd: d' then
        // 8 aligned words. The even block's first group joins q0,q1 with q30,q31.
        int off;
        if (blk % 2) off = 4 * ss + i;
        else if (ss == 0) { const int e[4] = {0, 1, 30, 31}; off = e[i]; }
        else off = 4 * ss - 2 + i;
        return 32 * blk + off;
    }
    // q4_0: a pair of blocks = 36 bytes = 9 words; byte j holds elements j (low nibble) and j+16 (high nibble).
    // Group (x0,x1,x2,x3) gives k-step 2g: lows (x0,x2 | x1,x3) and k-step 2g+1: highs.
    const int grp = ss / 2, hi = ss % 2;
    int j[4];
    if (blk % 2) { for (int u = 0; u < 4; u++) j[u] = 4 * grp + u; }
    else if (grp == 0) { j[0] = 0; j[1] = 1; j[2] = 14; j[3] = 15; }
    else { for (int u = 0; u < 4; u++) j[u] = 4 * grp - 2 + u; }
    const int order[4] = {j[0], j[2], j[1], j[3]};
    return 32 * blk + 16 * hi + order[i];
}

// P.V: lane g of the A fragment (V^T) holds two head-dim rows per m-tile mt: dV(mt, g, 0) (row g) and dV(mt, g, 1)
// (row g + 8). Lane g owns a contiguous byte range of one quant block.
__host__ __device__ inline int dV(int quant, int hd, int mt, int g, int half) {
    if (quant == 0) return 16 * mt + g + 8 * half;   // f16 rows: ldmatrix.trans fragments, natural order
    if (quant == 1) {
        const int base = hd == 128 ? 16 * g : 32 * g;
        return base + 2 * mt + half;
    }
    const int b = hd == 128 ? g / 2 : g;
    const int e0 = hd == 128 ? 8 * (g % 2) : 0;
    const int u = mt / 2, e = e0 + 2 * u;
    return 32 * b + e + (mt % 2 ? 16 : 0) + half;
}

// Int8-domain QK (QUANT 3): per quant block, lane t of a quad feeds k = 4t..4t+3 and 16+4t..16+4t+3 of the block's
// m16n8k32 MMA with two 4-byte words of each key row. A pair of Q8_0 blocks is 17 aligned words:
// (d,q0,q1)(q2..q5)...(q26..q29)(q30,q31,d') then the odd block's 8 words. i8_word(odd, t, w) is the byte offset in the
// pair of the lane's word w (0, 1); for the even block, lane 0's word 0 (d,q0,q1) is joined with the q30,q31 half of
// word 8 by one PRMT (selector 0x5432). i8_elem(odd, t, i) is the block element of byte i (0..7) of those two words, the
// order Q's int8 values take in the B fragment.
__host__ __device__ inline int i8_word(int odd, int t, int w) { return odd ? 36 + 8 * t + 4 * w : 8 * t + 4 * w; }
__host__ __device__ inline int i8_elem(int odd, int t, int i) {
    if (odd) return 8 * t + i;
    if (t == 0 && i < 4) return i < 2 ? i : 28 + i;   // (q0, q1, q30, q31)
    return 8 * t - 2 + i;
}

// ---------------------------------------------------------------- fragment builders
// 4 int8 values (one aligned word) -> two f16x2 of f16(d * q): (v0,v1) and (v2,v3)
__device__ __forceinline__ void q8_word(uint32_t w, uint32_t s2, uint32_t &lo, uint32_t &hi) {
    const uint32_t u = w ^ 0x80808080u;                       // q + 128
    const uint32_t magic = 0x64646464u;
    lo = hmul2(hsub2(prmt(u, magic, 0x4140u), 0x64806480u), s2);   // (1024 + u) - 1152 = q
    hi = hmul2(hsub2(prmt(u, magic, 0x4342u), 0x64806480u), s2);
}
// 4 bytes of q4_0 nibbles -> (x0.lo, x2.lo), (x1.lo, x3.lo), (x0.hi, x2.hi), (x1.hi, x3.hi) as f16x2 of f16(d*(n-8))
__device__ __forceinline__ void q4_word(uint32_t w, uint32_t s2, uint32_t &l02, uint32_t &l13, uint32_t &h02,
                                        uint32_t &h13) {
    const uint32_t m = 0x000F000Fu, magic = 0x64006400u, off = 0x64086408u;   // (1024 + n) - 1032 = n - 8
    l02 = hmul2(hsub2(and_or(w, m, magic), off), s2);
    l13 = hmul2(hsub2(and_or(w >> 8, m, magic), off), s2);
    h02 = hmul2(hsub2(and_or(w >> 4, m, magic), off), s2);
    h13 = hmul2(hsub2(and_or(w >> 12, m, magic), off), s2);
}

// ---------------------------------------------------------------- the kernel
// CTA x of the launch takes jobs x, x + gridDim.x, x + 2 gridDim.x, ... of p.jobs[0, p.n_jobs); the plans launch one
// CTA per job (measured faster than fewer CTAs taking several jobs each: the block scheduler balances the jobs). The
// stages of a CTA's jobs, in order, are one stream g = 0, 1, 2, ... through the ring: stage g lands in buffer
// g % NSTAGE, so the copies of a next job's first stages are in flight while the previous job's last stages are
// computed and its partial written.
template <int HD, int QUANT, int W>
__global__ void __launch_bounds__(32 * W, min_ctas(HD, W)) decode_kernel(const Params p) {
    constexpr int NMT = HD / 16;   // k-steps of QK^T = m-tiles of P.V
    constexpr int STAGE_KEYS = stage_keys(HD);
    constexpr int NSTAGE = nstage(HD);
    constexpr bool I8 = QUANT == 3;           // int8-domain QK over Q8_0 rows
    constexpr int QS = I8 ? 1 : QUANT;        // the rows' storage format
    constexpr int NBK = HD / 32;              // quant blocks in a head
    constexpr int GB = q_group_bytes(QS);
    constexpr int PAIR = 2 * GB;   // bytes of an aligned pair of quant blocks
    static_assert(STAGE_KEYS == TILE_KEYS, "a stage is one MMA tile of keys");

    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t row = p.row, gs = p.gs;
    const uint32_t half_stage = (STAGE_KEYS / 2) * gs;    // K pairs, then V pairs
    const uint32_t stage_bytes = 2u * half_stage;
    // shared-memory offset of key k of a stage (keys in pairs)
    auto kofs = [&](uint32_t k) -> uint32_t { return (k / 2) * gs + (k % 2) * row; };
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NSTAGE * stage_bytes + SMEM_SLACK);
    uint64_t *never = full + NSTAGE;   // completed by nobody: the stall test hook waits on it
    uint32_t *released = reinterpret_cast<uint32_t *>(never + 1);   // per buffer: warps done with it, ever
    uint32_t *issued = released + NSTAGE;                            // per buffer: the last stream stage issued into it
    volatile int *abort_flag = reinterpret_cast<volatile int *>(issued + NSTAGE);

    const uint32_t n_hgroups = p.nkv / p.hg;
    const uint32_t hgi = blockIdx.y % n_hgroups, rbi = blockIdx.y / n_hgroups;
    const uint32_t h0 = hgi * p.hg;
    const uint32_t rg0 = rbi * p.rgc;
    const uint32_t nrg = min(p.rgc, p.n_rg - rg0);
    const uint32_t n_active = p.hg * nrg;         // warps with work: one per (head, row group) stream
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t copy_bytes = (uint32_t) (p.hg * p.hb);
    constexpr uint32_t NEVER = 0xFFFFFFFFu;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; s++) { mbar_init(&full[s], 1); released[s] = 0; issued[s] = NEVER; }
        mbar_init(never, 1);
        // a CTA started after another one gave up a wait does no work (a systematic failure ends in one timeout)
        *abort_flag = *(volatile int *) p.status != ST_OK;
        fence_mbar_init();
    }
    __syncthreads();
    if (*abort_flag || warp >= n_active || blockIdx.x >= p.n_jobs) return;

    auto stages_of = [&](uint32_t jn) -> uint32_t { return (p.jobs[jn].nk + STAGE_KEYS - 1) / STAGE_KEYS; };
    // stage `it` of job `jn` as stream stage g, into buffer g % NSTAGE: K rows then V rows, one bulk copy per pair of
    // key rows (warp-collective)
    auto issue = [&](uint32_t jn, uint32_t it, uint32_t g) {
        const Job jb = p.jobs[jn];
        const uint32_t s = g % NSTAGE;
        const uint32_t valid = min((uint32_t) STAGE_KEYS, jb.nk - it * STAGE_KEYS);
        if (lane == 0) {
            issued[s] = g;
            mbar_arrive_expect_tx(&full[s], 2u * valid * copy_bytes);
        }
        __syncwarp();
        if (2 * lane < valid) {   // lane copies keys 2*lane, 2*lane+1 (one row if the stage ends there)
            const uint64_t off = (uint64_t) (jb.key0 + it * STAGE_KEYS + 2 * lane) * p.rs + h0 * p.hb;
            const uint8_t *kb = jb.k + off, *vb = jb.v + off;
            const bool two = 2 * lane + 1 < valid;
            uint8_t *dst = smem + s * stage_bytes + lane * gs;
            if (p.rs == copy_bytes) {   // the head group is the whole position: the pair is one contiguous range
                const uint32_t bytes = (two ? 2u : 1u) * copy_bytes;
                bulk_g2s(dst, kb, bytes, &full[s]);
                bulk_g2s(dst + half_stage, vb, bytes, &full[s]);
            } else {                    // a head group of a wider (or padded) position: one copy per row
                bulk_g2s(dst, kb, copy_bytes, &full[s]);
                bulk_g2s(dst + half_stage, vb, copy_bytes, &full[s]);
                if (two) {
                    bulk_g2s(dst + row, kb + p.rs, copy_bytes, &full[s]);
                    bulk_g2s(dst + half_stage + row, vb + p.rs, copy_bytes, &full[s]);
                }
            }
        }
    };
    // stream stage g + NSTAGE, found from the caller's place in the stream (job jc, which starts at stream stage g0 and
    // has nc stages): later in job jc, or in one of the CTA's next jobs (each has at least one stage)
    auto issue_ahead = [&](uint32_t jc, uint32_t g0, uint32_t nc, uint32_t g) {
        uint32_t target = g + NSTAGE - g0, jn = jc, n = nc;
        while (target >= n) {
            target -= n;
            jn += gridDim.x;
            if (jn >= p.n_jobs) return;
            n = stages_of(jn);
        }
        issue(jn, target, g + NSTAGE);
    };
    // after a wait gave up: every copy issued so far lands before the CTA exits (warp 0 waits for them, bounded)
    auto abort_and_drain = [&]() {
        if (lane == 0) {
            *abort_flag = 1;
            atomicCAS(p.status, ST_OK, ST_TIMEOUT_FULL);
        }
        if (warp == 0 && lane == 0) {
            const uint64_t drain_ns = p.timeout_ns > DRAIN_NS ? p.timeout_ns : DRAIN_NS;
            for (int s = 0; s < NSTAGE; s++) {
                const uint32_t gi = ((volatile uint32_t *) issued)[s];
                if (gi == NEVER) continue;
                if (!mbar_wait_bounded(&full[s], (gi / NSTAGE) & 1, drain_ns, nullptr))
                    atomicCAS(p.status, ST_OK, ST_TIMEOUT_DRAIN);
            }
        }
    };
    if (warp == 0) {   // the first NSTAGE stream stages
        uint32_t jn = blockIdx.x, it = 0, n = stages_of(jn);
        for (uint32_t g = 0; g < NSTAGE; g++) {
            issue(jn, it, g);
            if (++it == n) {
                it = 0;
                jn += gridDim.x;
                if (jn >= p.n_jobs) break;
                n = stages_of(jn);
            }
        }
    }

    // ------------------------------------------------ consumer warps
    const uint32_t hl = warp % p.hg, rgl = warp / p.hg;
    const uint32_t h = h0 + hl, rg = rg0 + rgl;
    const uint32_t g = lane / 4, t = lane % 4;
    const uint32_t hoff = hl * (uint32_t) p.hb;
    bool ok = true;
    if (p.stall && !mbar_wait_bounded(never, 0, p.timeout_ns, abort_flag)) ok = false;

    uint32_t gst = 0;   // stream stage
    for (uint32_t jc = blockIdx.x; ok && jc < p.n_jobs; jc += gridDim.x) {
    const Job job = p.jobs[jc];
    const uint32_t n_stages = (job.nk + STAGE_KEYS - 1) / STAGE_KEYS;
    const uint32_t g0 = gst;

    // Q fragments (B operand of S^T = K.Q^T): row n = g of this row group, k values permuted as dK
    uint32_t qf[I8 ? 1 : NMT][2];
    // int8-domain QK: Q's int8 words per quant block (k 4t.. and 16+4t.. of the block's MMA) and the block scales of
    // rows 2t, 2t+1 (the lane's accumulator columns)
    uint32_t qi[I8 ? NBK : 1][2];
    float dq[I8 ? NBK : 1][2];
    if constexpr (I8) {
        const uint32_t row = rg * 8 + g;
        const bool real = row < p.rows;
        const uint16_t *q = p.Qs + (((uint64_t) job.set * p.nkv + h) * p.rows + (real ? row : 0)) * HD;
#pragma unroll
        for (int b = 0; b < NBK; b++) {
            // the block's values in the order the K words of the lane give them (i8_elem)
            float x[8];
#pragma unroll
            for (int i = 0; i < 8; i++)
                x[i] = real ? __half2float(__ushort_as_half(q[32 * b + i8_elem(b % 2, (int) t, i)])) : 0.f;
            float am = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) am = fmaxf(am, fabsf(x[i]));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));   // the quad holds the row's 32 values
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
            const float df = __half2float(__float2half_rn(__fdiv_rn(am, 127.f)));
            const float id = df != 0.f ? __frcp_rn(df) : 0.f;
            uint32_t wv[2] = {0u, 0u};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int v = __float2int_rn(fmaxf(-127.f, fminf(127.f, __fmul_rn(x[i], id))));
                wv[i / 4] |= ((uint32_t) v & 0xFFu) << (8 * (i % 4));
            }
            qi[b][0] = wv[0];
            qi[b][1] = wv[1];
            dq[b][0] = __shfl_sync(0xffffffffu, df, 8 * t);       // row 2t lives in quad 2t
            dq[b][1] = __shfl_sync(0xffffffffu, df, 8 * t + 4);   // row 2t+1
        }
    } else {
        const uint32_t row = rg * 8 + g;
        const uint16_t *q = p.Qs + (((uint64_t) job.set * p.nkv + h) * p.rows + (row < p.rows ? row : 0)) * HD;
#pragma unroll
        for (int s = 0; s < NMT; s++) {
            uint16_t v[4];
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = row < p.rows ? q[dK(QUANT, s, t, i)] : (uint16_t) 0;
            qf[s][0] = (uint32_t) v[0] | ((uint32_t) v[1] << 16);
            qf[s][1] = (uint32_t) v[2] | ((uint32_t) v[3] << 16);
        }
    }

    float o[NMT][4];
#pragma unroll
    for (int mt = 0; mt < NMT; mt++) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    float m0 = M_EMPTY, m1 = M_EMPTY, l0 = 0.f, l1 = 0.f;   // rows 2t, 2t+1 of the 8-row group
    // Lazy running max: P is taken against a reference max mb (log2 units) that moves only when a score exceeds it by
    // more than LAZY_T (P <= 2^LAZY_T, well inside f16), so most tiles skip the cross-lane max and the O rescale. The
    // exact maximum (ml, lane-local then reduced) is restored at the end of the job: O and l are rescaled to it once.
    constexpr float LAZY_T = 8.f;
    float mb0 = M_EMPTY * LOG2E, mb1 = M_EMPTY * LOG2E;
    float th0 = M_EMPTY, th1 = M_EMPTY;        // scores (natural units) above these move mb
    float ml0 = -INFINITY, ml1 = -INFINITY;    // lane-local maxima of the scores

    for (uint32_t it = 0; it < n_stages; it++, gst++) {
        const uint32_t s = gst % NSTAGE;
        if (!mbar_wait_bounded(&full[s], (gst / NSTAGE) & 1, p.timeout_ns, abort_flag)) { ok = false; break; }
        const uint32_t valid = min((uint32_t) STAGE_KEYS, job.nk - it * STAGE_KEYS);
        const uint32_t kbase = smem_u32(smem + s * stage_bytes) + hoff;
        const uint32_t vbase = kbase + half_stage;
        for (uint32_t tt = 0; tt < STAGE_KEYS / TILE_KEYS; tt++) {
            const int tvalid = (int) valid - (int) tt * TILE_KEYS;
            if (tvalid <= 0) break;
            const uint32_t tk = kbase + tt * (TILE_KEYS / 2) * gs;   // the tile's 8 pairs
            const uint32_t tv = vbase + tt * (TILE_KEYS / 2) * gs;

            // ---- S^T = K . Qs^T  (lane: keys g, g+8; its quant block(s) t (+4))
            float c[4] = {0.f, 0.f, 0.f, 0.f};
            if constexpr (QS == 0) {
                // f16 rows: ldmatrix.x4 gives each k-step's A fragment (matrices: keys 2r | 2r+1 x d +0 | +8)
                const uint32_t r = lane % 8, mi = lane / 8;
                const uint32_t ka = tk + kofs(2 * r + (mi & 1)) + (mi >> 1) * 16;
#pragma unroll
                for (int ks = 0; ks < NMT; ks++) {
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(ka + 32 * ks, a0, a1, a2, a3);
                    mma16816(c, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
                }
            } else if constexpr (I8) {
                // per block the lane takes 2 words of keys g and g+8 (i8_word), one s8 MMA gives the block's T, and
                // the scores take float(T) * (dq * dk) in block order
#pragma unroll
                for (int j = 0; j < NBK / 2; j++) {
                    const uint32_t pb = (uint32_t) (PAIR * j);
                    uint32_t ea[2], eb[2], oa[2], ob[2];
                    float dke[2], dko[2];
#pragma unroll
                    for (int kk = 0; kk < 2; kk++) {
                        const uint32_t rk = tk + kofs(2 * g + kk) + pb;   // MMA rows g, g+8
                        const uint32_t w0 = lds32o<0>(rk), w8 = lds32o<32>(rk);
                        ea[kk] = prmt(lds32(rk + i8_word(0, (int) t, 0)), w8, t == 0 ? 0x5432u : 0x3210u);
                        eb[kk] = lds32(rk + i8_word(0, (int) t, 1));
                        oa[kk] = lds32(rk + i8_word(1, (int) t, 0));
                        ob[kk] = lds32(rk + i8_word(1, (int) t, 1));
                        dke[kk] = h2f_bits(w0);
                        dko[kk] = h2f_bits(w8 >> 16);
                    }
                    int T[4];
                    mma16832_s8(T, ea[0], ea[1], eb[0], eb[1], qi[2 * j][0], qi[2 * j][1]);
                    c[0] = fmaf(__int2float_rn(T[0]), __fmul_rn(dq[2 * j][0], dke[0]), c[0]);
                    c[1] = fmaf(__int2float_rn(T[1]), __fmul_rn(dq[2 * j][1], dke[0]), c[1]);
                    c[2] = fmaf(__int2float_rn(T[2]), __fmul_rn(dq[2 * j][0], dke[1]), c[2]);
                    c[3] = fmaf(__int2float_rn(T[3]), __fmul_rn(dq[2 * j][1], dke[1]), c[3]);
                    mma16832_s8(T, oa[0], oa[1], ob[0], ob[1], qi[2 * j + 1][0], qi[2 * j + 1][1]);
                    c[0] = fmaf(__int2float_rn(T[0]), __fmul_rn(dq[2 * j + 1][0], dko[0]), c[0]);
                    c[1] = fmaf(__int2float_rn(T[1]), __fmul_rn(dq[2 * j + 1][1], dko[0]), c[1]);
                    c[2] = fmaf(__int2float_rn(T[2]), __fmul_rn(dq[2 * j + 1][0], dko[1]), c[2]);
                    c[3] = fmaf(__int2float_rn(T[3]), __fmul_rn(dq[2 * j + 1][1], dko[1]), c[3]);
                }
            } else {
#pragma unroll
            for (int rep = 0; rep < HD / 128; rep++) {
                const int blk = t + 4 * rep;
                const uint32_t odd = blk % 2;
                const uint32_t pb = (uint32_t) (PAIR * (blk / 2));
                // the lane's words: NWK-1 "slots" of its values, then the pair's shared word (even block: its last
                // values; odd block: its scale). Even block: slots = pair words 0..NWK-2; odd block: the NWK-1 aligned
                // words after the shared one. One lane-dependent PRMT selector then serves both parities.
                constexpr int NWK = QUANT == 1 ? 9 : 5;
                const uint32_t ssel = odd ? 0x7676u : 0x1010u;   // scale: odd -> shared word bytes 2-3, even -> slot 0 bytes 0-1
                const uint32_t gsel = odd ? 0x3210u : 0x5432u;   // group 0: odd -> slot 0, even -> (v0, v1 | v30, v31)
                uint32_t w[2][NWK], s2[2], g0[2];
#pragma unroll
                for (int kk = 0; kk < 2; kk++) {
                    const uint32_t rk = tk + kofs(2 * g + kk) + pb;   // MMA rows g, g+8
                    const uint32_t rb = rk + (odd ? 4u * NWK : 0u);
                    w[kk][0] = lds32o<0>(rb);
                    w[kk][1] = lds32o<4>(rb);
                    w[kk][2] = lds32o<8>(rb);
                    w[kk][3] = lds32o<12>(rb);
                    if (NWK > 5) {
                        w[kk][4 % NWK] = lds32o<16>(rb);
                        w[kk][5 % NWK] = lds32o<20>(rb);
                        w[kk][6 % NWK] = lds32o<24>(rb);
                        w[kk][7 % NWK] = lds32o<28>(rb);
                    }
                    w[kk][NWK - 1] = lds32o<4 * (NWK - 1)>(rk);
                    s2[kk] = prmt(w[kk][0], w[kk][NWK - 1], ssel);
                    g0[kk] = prmt(w[kk][0], w[kk][NWK - 1], gsel);
                }
                if (QUANT == 1) {
#pragma unroll
                    for (int ss = 0; ss < 8; ss++) {
                        uint32_t lo[2], hi[2];
#pragma unroll
                        for (int kk = 0; kk < 2; kk++) q8_word(ss == 0 ? g0[kk] : w[kk][ss], s2[kk], lo[kk], hi[kk]);
                        const int sidx = 8 * rep + ss;
                        mma16816(c, lo[0], lo[1], hi[0], hi[1], qf[sidx][0], qf[sidx][1]);
                    }
                } else {
#pragma unroll
                    for (int gi = 0; gi < 4; gi++) {
                        uint32_t l02[2], l13[2], h02[2], h13[2];
#pragma unroll
                        for (int kk = 0; kk < 2; kk++) {
                            q4_word(gi == 0 ? g0[kk] : w[kk][gi], s2[kk], l02[kk], l13[kk], h02[kk], h13[kk]);
                        }
                        const int sidx = 8 * rep + 2 * gi;
                        mma16816(c, l02[0], l02[1], l13[0], l13[1], qf[sidx][0], qf[sidx][1]);
                        mma16816(c, h02[0], h02[1], h13[0], h13[1], qf[sidx + 1][0], qf[sidx + 1][1]);
                    }
                }
            }
            }

            // ---- V words of the tile, loaded before the softmax so that their latency hides under it
            // k indices 2t, 2t+1, 2t+8, 2t+9 are MMA rows of S^T, i.e. keys 4t, 4t+2, 4t+1, 4t+3
            const uint32_t key[4] = {4 * t, 4 * t + 2, 4 * t + 1, 4 * t + 3};
            // the lane's data bytes start 2 bytes into a word for even quant blocks: load the covering words and
            // shift them into alignment (funnel shift by 8*sig bits; sig is 0 or 2), so every later index is static
            // (f16 rows: the P.V fragments come from ldmatrix.trans in the P.V loop instead)
            constexpr int NB = QS == 1 ? (HD == 128 ? 16 : 32) : QS == 2 ? (HD == 128 ? 8 : 16) : 4;   // bytes per lane per key
            constexpr int NW = NB / 4;
            uint32_t VW[4][NW];
            uint32_t s01 = 0, s23 = 0;
            if constexpr (QS != 0) {
            const int b = HD == 128 ? (int) g / 2 : (int) g;
            const int hh = HD == 128 ? (int) g % 2 : 0;
            const uint32_t pb = (uint32_t) (PAIR * (b / 2));
            const uint32_t start = QS == 1 ? pb + ((b % 2) ? 36u : 2u) + 16u * hh : pb + ((b % 2) ? 20u : 2u) + 8u * hh;
            const uint32_t sig = start % 4, wa = start - sig, shift = 8 * sig;
            const uint32_t soff = pb + ((b % 2) ? (uint32_t) GB : 0u);
            uint32_t sc[4];
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const uint32_t rb = tv + kofs(key[kk]);
                sc[kk] = lds16(rb + soff);
                uint32_t raw[NW + 1];
                const uint32_t ra = rb + wa;
                raw[0] = lds32o<0>(ra);
                raw[1] = lds32o<4>(ra);
                if (NW > 2) { raw[2 % (NW + 1)] = lds32o<8>(ra); raw[3 % (NW + 1)] = lds32o<12>(ra); }
                if (NW > 4) {
                    raw[4 % (NW + 1)] = lds32o<16>(ra); raw[5 % (NW + 1)] = lds32o<20>(ra);
                    raw[6 % (NW + 1)] = lds32o<24>(ra); raw[7 % (NW + 1)] = lds32o<28>(ra);
                }
                raw[NW] = sig ? lds32(ra + 4 * NW) : 0u;
#pragma unroll
                for (int i = 0; i < NW; i++) VW[kk][i] = __funnelshift_r(raw[i], raw[i + 1], shift);
            }
            // keys past the stage's valid count hold whatever the buffer held before (possibly never written):
            // a zero scale makes their V exactly 0, so P = 0 times it cannot produce NaN
            if (tvalid < TILE_KEYS) {
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                    if ((int) key[kk] >= tvalid) sc[kk] = 0u;
            }
            // key pairs: (key0,key1) -> a0/a1, (key2,key3) -> a2/a3
            s01 = sc[0] | (sc[1] << 16);
            s23 = sc[2] | (sc[3] << 16);
            }

            // ---- online softmax over this tile (rows 2t, 2t+1; keys g, g+8) against the lazy reference max
            if (tvalid < TILE_KEYS) {
                if ((int) (2 * g) >= tvalid) c[0] = c[1] = -INFINITY;       // row g = key 2g
                if ((int) (2 * g + 1) >= tvalid) c[2] = c[3] = -INFINITY;   // row g+8 = key 2g+1
            }
            float mx0 = fmaxf(c[0], c[2]), mx1 = fmaxf(c[1], c[3]);
            ml0 = fmaxf(ml0, mx0);
            ml1 = fmaxf(ml1, mx1);
            if (__any_sync(0xffffffffu, mx0 > th0 || mx1 > th1)) {
#pragma unroll
                for (int x = 4; x < 32; x <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, x));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, x));
                }
                const float nb0 = fmaxf(mb0, mx0 * LOG2E), nb1 = fmaxf(mb1, mx1 * LOG2E);
                const float al0 = ex2(mb0 - nb0), al1 = ex2(mb1 - nb1);
                l0 *= al0;
                l1 *= al1;
#pragma unroll
                for (int mt = 0; mt < NMT; mt++) { o[mt][0] *= al0; o[mt][1] *= al1; o[mt][2] *= al0; o[mt][3] *= al1; }
                mb0 = nb0;
                mb1 = nb1;
                th0 = (mb0 + LAZY_T) * (1.f / LOG2E);
                th1 = (mb1 + LAZY_T) * (1.f / LOG2E);
            }
            const float p0 = ex2(fmaf(c[0], LOG2E, -mb0)), p1 = ex2(fmaf(c[1], LOG2E, -mb1));
            const float p2 = ex2(fmaf(c[2], LOG2E, -mb0)), p3 = ex2(fmaf(c[3], LOG2E, -mb1));
            l0 += p0 + p2;
            l1 += p1 + p3;
            const uint32_t pb0 = movtrans(pack_h2(p0, p1));   // P^T keys 2t,2t+1 for row g
            const uint32_t pb1 = movtrans(pack_h2(p2, p3));   // keys 2t+8, 2t+9

            // ---- O^T += V^T . P^T  (lane: keys 2t,2t+1,2t+8,2t+9; head-dim rows dV(mt, g, 0/1))
            {
                if constexpr (QS == 0) {
                    // f16 rows: ldmatrix.x4.trans gives each m-tile's A fragment (matrices: keys 2r | 2r+1 of the P^T
                    // order x d +0 | +8); keys past the stage's valid count are zeroed in the fragment (their rows
                    // may hold anything, and 0 * NaN would poison O)
                    const uint32_t r = lane % 8, mi = lane / 8;
                    const uint32_t va = tv + kofs(2 * r + (mi >> 1)) + (mi & 1) * 16;
                    uint32_t m01 = 0xFFFFFFFFu, m23 = 0xFFFFFFFFu;
                    if (tvalid < TILE_KEYS) {
                        m01 = ((int) key[0] < tvalid ? 0x0000FFFFu : 0u) | ((int) key[1] < tvalid ? 0xFFFF0000u : 0u);
                        m23 = ((int) key[2] < tvalid ? 0x0000FFFFu : 0u) | ((int) key[3] < tvalid ? 0xFFFF0000u : 0u);
                    }
#pragma unroll
                    for (int mt = 0; mt < NMT; mt++) {
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4_t(va + 32 * mt, a0, a1, a2, a3);
                        mma16816(o[mt], a0 & m01, a1 & m01, a2 & m23, a3 & m23, pb0, pb1);
                    }
                } else if constexpr (QS == 1) {
#pragma unroll
                    for (int mt = 0; mt < NMT; mt++) {
                        constexpr uint32_t SEL[2] = {0x5140u, 0x7362u};   // (a.e, b.e, a.e+1, b.e+1), e = 2mt
                        const int wi = mt / 2;
                        uint32_t lo01, hi01, lo23, hi23;
                        q8_word(prmt(VW[0][wi], VW[1][wi], SEL[mt % 2]), s01, lo01, hi01);
                        q8_word(prmt(VW[2][wi], VW[3][wi], SEL[mt % 2]), s23, lo23, hi23);
                        mma16816(o[mt], lo01, hi01, lo23, hi23, pb0, pb1);
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < NMT / 2; u++) {
                        constexpr uint32_t SEL[2] = {0x5410u, 0x7632u};   // (a.e, a.e+1, b.e, b.e+1), e = 2u
                        const int wi = u / 2;
                        uint32_t a_l0, a_l1, a_h0, a_h1, c_l0, c_l1, c_h0, c_h1;
                        // q4_word on an interleaved word: l02 = byte e low nibble (keys a,b), l13 = byte e+1 low,
                        // h02 = byte e high, h13 = byte e+1 high
                        q4_word(prmt(VW[0][wi], VW[1][wi], SEL[u % 2]), s01, a_l0, a_l1, a_h0, a_h1);
                        q4_word(prmt(VW[2][wi], VW[3][wi], SEL[u % 2]), s23, c_l0, c_l1, c_h0, c_h1);
                        mma16816(o[2 * u], a_l0, a_l1, c_l0, c_l1, pb0, pb1);       // rows g <- e, g+8 <- e+1
                        mma16816(o[2 * u + 1], a_h0, a_h1, c_h0, c_h1, pb0, pb1);   // rows g <- e+16, g+8 <- e+17
                    }
                }
            }
        }
        // release the buffer; the last warp to do so refills it with stream stage gst + NSTAGE
        __syncwarp();
        uint32_t last = 0;
        if (lane == 0) {
            __threadfence_block();   // this warp's reads of the buffer are ordered before its count
            last = (atomicAdd(&released[s], 1u) + 1u) % n_active == 0;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            fence_proxy_async();     // ... and before the bulk copies (async proxy) that overwrite it
            issue_ahead(jc, g0, n_stages, gst);
        }
    }
    if (!ok) break;

    // ---- report the exact maximum of each row: rescale O and l from the lazy reference max to it (an empty row keeps
    // m = M_EMPTY, l = 0)
#pragma unroll
    for (int x = 4; x < 32; x <<= 1) {
        ml0 = fmaxf(ml0, __shfl_xor_sync(0xffffffffu, ml0, x));
        ml1 = fmaxf(ml1, __shfl_xor_sync(0xffffffffu, ml1, x));
    }
    {
        const float f0 = ml0 > -INFINITY ? ex2(mb0 - ml0 * LOG2E) : 1.f;
        const float f1 = ml1 > -INFINITY ? ex2(mb1 - ml1 * LOG2E) : 1.f;
        l0 *= f0;
        l1 *= f1;
#pragma unroll
        for (int mt = 0; mt < NMT; mt++) { o[mt][0] *= f0; o[mt][1] *= f1; o[mt][2] *= f0; o[mt][3] *= f1; }
        m0 = ml0 > -INFINITY ? ml0 : M_EMPTY;
        m1 = ml1 > -INFINITY ? ml1 : M_EMPTY;
    }
    // l summed over the lanes of a row (keys g)
#pragma unroll
    for (int x = 4; x < 32; x <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, x);
        l1 += __shfl_xor_sync(0xffffffffu, l1, x);
    }

    // ---- write the job's slot partial
    const uint64_t rbase = ((uint64_t) job.slot * p.nkv + h) * p.rows;
    const uint32_t r0 = rg * 8 + 2 * t, r1 = r0 + 1;
#pragma unroll
    for (int mt = 0; mt < NMT; mt++) {
        const int d0 = dV(QS, HD, mt, (int) g, 0), d1 = dV(QS, HD, mt, (int) g, 1);
        if (r0 < p.rows) {
            p.Op[(rbase + r0) * HD + d0] = o[mt][0];
            p.Op[(rbase + r0) * HD + d1] = o[mt][2];
        }
        if (r1 < p.rows) {
            p.Op[(rbase + r1) * HD + d0] = o[mt][1];
            p.Op[(rbase + r1) * HD + d1] = o[mt][3];
        }
    }
    if (g == 0) {
        if (r0 < p.rows) { p.Mp[rbase + r0] = l0 > 0.f ? m0 : -INFINITY; p.Lp[rbase + r0] = l0; }
        if (r1 < p.rows) { p.Mp[rbase + r1] = l1 > 0.f ? m1 : -INFINITY; p.Lp[rbase + r1] = l1; }
    }
    }   // jobs
    if (!ok) abort_and_drain();
}

}  // namespace dec
}  // namespace pa
