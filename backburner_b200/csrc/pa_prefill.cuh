// pa_prefill.cuh - partial attention for many query rows per KV head (prefill / ATTN_BIG calls, long verify
// batches) on the 5th-generation tensor cores: tcgen05.mma with accumulators in tensor memory (TMEM).
//
// Reference semantics: pa_attn_big (phone-attn/pa-metal.mm:379-487), the dense-row kernel the reference runs for
// prefill: rows of all groups of one KV head packed back to back, K/V blocks dequantised to f16, S = Qs.K^T and
// O += P.V on the matrix units with fp32 accumulation, online softmax over the valid keys (pa-metal.mm:452-464),
// one unnormalised (O, m, l) per chunk of keys. Head dim 128.
//
// One CTA = one chunk of keys of one segment x one KV head x NT tiles of 128 query rows. Warp roles:
//   warp 0             TMA: with two tiles the Q tiles once (128-byte swizzle, the UMMA operand layout), then per
//                      block (B keys: 128 with one tile at head dim 128, else 64) the raw quantised rows of this head (a
//                      16-byte-aligned window of each key row, 2-D tensor copies of 64 rows for K and for V; keys past
//                      the end read as zeros)
//   warps 1, 2         warp 1 allocates TMEM (512 columns: per tile S B columns, two P buffers of B / 2, O D; one tile:
//                      the Q tile too); one thread of warp 1 issues the S_t = Q_t K^T MMAs (M=128, N=B; A = Q from
//                      shared or, one tile, tensor memory) into S, one of warp 2 the O_t += P_t V MMAs (M=128, N=D,
//                      A = P read from TMEM, B = V read MN-major) into O
//   warps 4 .. 4+4NT   one warpgroup per Q tile: thread = query row = TMEM lane. Reads its row of S (B keys; S is
//                      free again once read), masks tail keys, online softmax in the log2 domain with lazy rescaling (the
//                      running max moves only when a block's max exceeds it by more than 8, so O in TMEM is rescaled
//                      rarely), writes P as packed f16 into the block's P buffer: the softmax never waits for a P.V
//                      except to rescale. With one tile the warpgroup also writes the Q tile into tensor memory
//   last 8 (NT = 1) or  dequantise each raw K and V block into f16 operand tiles (f16(d * q), 128-byte swizzle)
//   4 (NT = 2) warps
// All waits are bounded; a wait that runs out records a status, and every role still reaches the final barrier so
// TMEM is released.
#pragma once
#include <cuda.h>

#include "pa_common.cuh"
#include "pa_decode.cuh"

namespace pa {
namespace pre {

constexpr int HD = 128;
constexpr int BM = 128;   // query rows per tile = TMEM lanes
constexpr int BN = 64;    // keys per block
constexpr int NS = 3;     // raw stages of the CTA-pair kernel's TMA ring

// bytes of the 16-byte-aligned window that holds one head of a key row: the head (hd/32 blocks of 34 B for Q8_0, 18 B
// for Q4_0) plus its offset inside the window (head h starts at h * hb: offset 0 or 8 when hb % 16 == 8, else 0),
// rounded up to 16 (hd 128: 144 / 80; hd 256: 272 / 144)
__host__ __device__ constexpr int raw_row_bytes(int quant, int hd = 128) {
    return ((hd / 32) * (quant == 1 ? 34 : 18) + (((hd / 32) * (quant == 1 ? 34 : 18)) % 16 ? 8 : 0) + 15) / 16 * 16;
}

struct Params {
    const dec::Job *jobs;
    const uint16_t *Qs;           // f16(q*scale) [n_sets][nkv][rows][HD] (the one-tile kernel reads its rows directly)
    const CUtensorMap *kv_maps;   // [2*seg] K rows, [2*seg+1] V rows: 16-bit elements {rs/2, nk}, box {raw_row_bytes/2,
                                  // keys per copy} (16-bit elements keep a 272-byte window within TMA's 256-element box)
    float *Op, *Mp, *Lp;          // slot partials [slot][nkv][rows][HD], [slot][nkv][rows]
    int *status;
    uint64_t rs, hb;
    uint32_t nkv, rows, n_rt;     // n_rt: groups of NT*BM rows per head
    uint64_t timeout_ns;
    int stall;                    // test hook: the softmax warps first wait on a barrier that nothing completes (bounded)
};

// ---------------------------------------------------------------- tcgen05 / TMA helpers
__device__ __forceinline__ void tma_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// (volatile keeps it in order with the mbarrier waits, fences and commits around it, which all are volatile asm; no
// "memory" clobber, so the compiler need not re-read spilled or cached values around each issue)
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc));
}
// the same with A (M=128 x K=16, 16-bit, two per 32-bit column, row = lane) read from tensor memory
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc));
}
// 32 consecutive fp32 columns of this warp's 32 TMEM lanes: thread i gets lane (quarter*32 + i)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes from packed words (f16x2)
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// fp32 pairs (sm_100 .f32x2 arithmetic) and the three-input max
__device__ __forceinline__ uint64_t pack_f2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void unpack_f2(uint64_t x, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// 2^t0, 2^t1 on the FMA pipe (relieves the MUFU unit, which the softmax's exp2 keeps busy): t = n + f with n = rint(t)
// by the 1.5 * 2^23 addition trick, 2^f on [-0.5, 0.5] by a degree-3 polynomial least-squares fitted for this kernel
// (max relative error 7.5e-5, below P's f16 rounding), and n added to the result's exponent field by one integer
// multiply-add. Inputs below -125 give 2^-125 (P rounds to 0 in f16, and the row sum changes by < 1e-37).
__device__ __forceinline__ void ex2_pair_fma(float t0, float t1, float &p0, float &p1) {
    const uint64_t xa = pack_f2(fmaxf(t0, -125.f), fmaxf(t1, -125.f));
    const uint64_t tt = add_f2(xa, pack_f2(12582912.f, 12582912.f));
    float r0, r1, u0, u1;
    unpack_f2(add_f2(tt, pack_f2(-12582912.f, -12582912.f)), r0, r1);
    const uint64_t fv = add_f2(xa, pack_f2(-r0, -r1));
    uint64_t pp = fma_f2(pack_f2(0.0551716648f, 0.0551716648f), fv, pack_f2(0.2426111251f, 0.2426111251f));
    pp = fma_f2(pp, fv, pack_f2(0.6932609677f, 0.6932609677f));
    pp = fma_f2(pp, fv, pack_f2(0.9999280572f, 0.9999280572f));
    unpack_f2(pp, u0, u1);
    unpack_f2(tt, r0, r1);
    p0 = __uint_as_float(__float_as_uint(r0) * 0x800000u + __float_as_uint(u0));
    p1 = __uint_as_float(__float_as_uint(r1) * 0x800000u + __float_as_uint(u1));
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void lds128(uint32_t addr, uint32_t &a, uint32_t &b, uint32_t &c, uint32_t &d) {
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr));
}

// UMMA shared-memory descriptor, 128-byte swizzle (sm100 layout: start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46),
// version 1 at bit 46, layout type 2 = SWIZZLE_128B at bits [61,64))
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((saddr >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A/B f16 (0), A K-major, B K- or MN-major (bit 16),
// N>>3 at bits 17-22, M>>4 at bits 24-28
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int b_mn_major) {
    return (1u << 4) | ((uint32_t) b_mn_major << 16) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (M >> 4) << 24);
}

// The single-CTA kernel's layout depends on the tile count NT and the head dim D (D = 256: one tile only, the reference
// server's wire geometry).
// keys per block: 128 with one tile at D = 128 (a block's hand-offs between the roles cost about the same whatever its
// size, so larger blocks amortise them), else 64 (D = 256: the same bytes per block)
__host__ __device__ constexpr int block_keys(int nt, int d = 128) { return nt == 1 && d == 128 ? 128 : 64; }
// dequantised K and V buffers (a ring of 2: 32 KB each with one tile)
__host__ __device__ constexpr int kv_bufs(int nt, int d = 128) { return 2; }
// raw (quantised) K/V stages of the TMA ring: 3 with two tiles, else 2 (a stage of Q8_0 rows is 34-36 KB)
__host__ __device__ constexpr int raw_stages(int quant, int nt, int d = 128) {
    return d == 128 && block_keys(nt, d) == 64 ? 3 : 2;
}
// dequant warps of the single-CTA kernel: 8 with one Q tile (the dequant is the larger cost per row there), 4 with two
__host__ __device__ constexpr int dq_warps(int nt) { return nt == 1 ? 8 : 4; }
// warps of a CTA: TMA + MMA warpgroup, one softmax warpgroup per Q tile, dequant
__host__ __device__ constexpr int cta_warps(int nt) { return 4 + 4 * nt + dq_warps(nt); }
// S accumulators per Q tile in tensor memory: one (each layout fills the 512 columns with S, P, O and Q; with a row's
// scores in registers S is free as soon as the softmax has read it)
__host__ __device__ constexpr int s_bufs(int nt, int d = 128) { return 1; }
// Q in tensor memory: the one-tile kernel keeps its Q tile in TMEM (D / 2 columns) as the A operand of S = Q K^T, so an S
// MMA reads only its K slice from shared memory (from shared memory, each N = 64 MMA re-read a 4 KB Q slice: twice the
// K bytes it multiplies); with two tiles tensor memory is full and Q stays in shared memory
__host__ __device__ constexpr bool q_in_tmem(int nt) { return nt == 1; }
// P buffers per Q tile in tensor memory: two (the softmax writes P of block j once P.V of block j-2 is done)
__host__ __device__ constexpr int p_bufs(int nt, int d = 128) { return 2; }

// shared-memory map (all operand tiles 1024-aligned); KVB dequantised K and V buffers
template <int QUANT, int NT, int D = 128>
struct Smem {
    static_assert(D == 128 || (D == 256 && NT == 1), "head dim 256 takes one Q tile");
    static constexpr int KVB = kv_bufs(NT, D);
    static constexpr int B = block_keys(NT, D);                    // keys per block
    static constexpr int RAWB = raw_row_bytes(QUANT, D);
    static constexpr int Q = 0;                                   // NT x [D/64 atom cols][128 rows][128 B] (or none)
    static constexpr int K = Q + (q_in_tmem(NT) ? 0 : NT * BM * D * 2);   // KVB x [D/64 atom cols][B keys][128 B]
    static constexpr int V = K + KVB * B * D * 2;                  // KVB x same (read MN-major)
    static constexpr int NRS = raw_stages(QUANT, NT, D);
    static constexpr int RAW = V + KVB * B * D * 2;                // NRS x (K rows, V rows) x [B][RAWB]
    static constexpr int RAW_STAGE = (2 * B * RAWB + 1023) / 1024 * 1024;
    static constexpr int BAR = RAW + NRS * RAW_STAGE;
    static constexpr int N_BAR = 1 + 2 * NRS + 4 * KVB + (2 * s_bufs(NT, D) + 2 * p_bufs(NT, D) + 1) * NT + 1 + 1;
    static constexpr int TOTAL = BAR + N_BAR * 8 + 32;
};

template <int QUANT, int NT, int D = 128>
__global__ void __launch_bounds__(32 * cta_warps(NT), 1) prefill_kernel(const __grid_constant__ CUtensorMap tq,
                                                                       const Params p) {
    using L = Smem<QUANT, NT, D>;
    constexpr int KVB = L::KVB;
    constexpr int B = L::B;   // keys per block
    constexpr int RAWB = L::RAWB;
    constexpr int GB = dec::q_group_bytes(QUANT);
    constexpr uint32_t IDESC_S = idesc_f16(BM, B, 0);
    constexpr uint32_t IDESC_PV = idesc_f16(BM, D, 1);
    // warpgroups: 0 = TMA (warp 0) + MMA (warps 1, 2) + 1 idle warp, 1..NT = softmax of tile t, last = dequant
    constexpr int SM0 = 4, DQ0 = 4 + 4 * NT;   // first softmax warp, first dequant warp
    constexpr int NDQ = dq_warps(NT);
    // tensor memory (512 columns) of tile t from column t * 256: S (B columns), two P buffers (B / 2 columns each, f16
    // packed two keys per column), O (D columns); one tile: Q at 384 (D / 2 columns). One tile at D = 128 (128-key
    // blocks): S 0-127, P 128 / 192, O 256-383; D = 256: S 0-63, P 64 / 96, O 128-383
    constexpr int NSB = s_bufs(NT, D), NPB = p_bufs(NT, D);
    constexpr bool QT = q_in_tmem(NT);
    constexpr uint32_t T_P = B, T_O = 2 * B, TCOLS = 512;
    constexpr uint32_t T_Q = 384;   // Q (one tile): row = lane, column c = f16 elements 2c, 2c + 1
    static_assert(NSB == 1 && NPB == 2 && T_O + D <= (NT == 1 ? T_Q : 256u) && T_Q + (QT ? D / 2 : 0) <= TCOLS,
                  "tensor memory layout");
    static_assert(!QT || NT == 1, "Q in tensor memory with one tile only");
    // column of P buffer i (relative to the tile)
    auto p_col = [](uint32_t i) -> uint32_t { return T_P + i * (B / 2); };

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // operand tiles need 1024-byte alignment (128-byte swizzle atoms): align the dynamic base explicitly
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const uint32_t sbase = smem_u32(smem);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L::BAR);
    uint64_t *q_full = bar;   // Q tile(s) in shared memory (TMA) or, one tile, in tensor memory (the softmax warps)
    constexpr int NRS = L::NRS;
    uint64_t *raw_full = bar + 1, *raw_empty = raw_full + NRS;
    uint64_t *k_full = raw_empty + NRS, *k_free = k_full + KVB, *v_full = k_free + KVB, *v_free = v_full + KVB;
    uint64_t *s_full = v_free + KVB;           // [NT][NSB]: S of the block in S buffer j % NSB of the tile
    uint64_t *s_empty = s_full + NT * NSB;     // [NT][NSB]: the softmax has read that S into registers
    uint64_t *p_full = s_empty + NT * NSB;     // [NT][NPB]: P of the block in P buffer j % NPB (one barrier per buffer,
                                               // so the softmax finishing a later block cannot complete block j's phase)
    uint64_t *pv_free = p_full + NPB * NT;     // [NT][NPB]: P.V of a block with P buffer i completed
    uint64_t *o_ready = pv_free + NPB * NT;    // [NT]: the last P.V completed (once)
    uint64_t *mma_done = o_ready + NT;         // every MMA this CTA issued has completed (before TMEM is freed)
    uint64_t *never = mma_done + 1;            // completed by nobody: the stall test hook waits on it
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + L::N_BAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    // CTA order (a 1-D grid): row-tile group fastest, then KV head, then job, so the CTAs that read the same K/V
    // blocks (all row groups and heads of one chunk of keys) run at the same time and share them through L2
    const uint32_t cid = blockIdx.x;
    const uint32_t rt = cid % p.n_rt, h = (cid / p.n_rt) % p.nkv;
    const dec::Job job = p.jobs[cid / (p.n_rt * p.nkv)];
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t nblk = (job.nk + B - 1) / B;
    const uint32_t hbyte = h * (uint32_t) p.hb;
    const int hx = (int) (hbyte & ~15u);          // window start (16-byte aligned) of this head in a key row
    const uint32_t hoff = hbyte & 15u;            // head start inside the window
    const uint32_t row0 = rt * NT * BM;           // first query row of this CTA (within the head)
    const uint64_t tmo = p.timeout_ns;
    bool ok = true;

    if (threadIdx.x == 0) {
        // Q in tensor memory: one arrival per softmax warp with a real row (see below), else the TMA thread's
        mbar_init(q_full, QT ? min(4u, (p.rows - row0 + 31) / 32) : 1u);
        for (int s = 0; s < NRS; s++) { mbar_init(&raw_full[s], 1); mbar_init(&raw_empty[s], NDQ); }
        for (int b = 0; b < KVB; b++) {
            mbar_init(&k_full[b], NDQ); mbar_init(&k_free[b], 1); mbar_init(&v_full[b], NDQ); mbar_init(&v_free[b], 1);
        }
        for (int t = 0; t < NT; t++) {
            // softmax warps that take part: those with a real row (a lane quarter wholly past the call's rows sits out;
            // NT = 1 only, see the softmax role)
            const uint32_t first = row0 + t * BM;
            const uint32_t nq = NT == 1 ? min(4u, (p.rows - first + 31) / 32) : 4u;
            for (int sb = 0; sb < NSB; sb++) {
                mbar_init(&s_full[t * NSB + sb], 1);
                mbar_init(&s_empty[t * NSB + sb], nq);
            }
            for (int i = 0; i < NPB; i++) {
                mbar_init(&p_full[t * NPB + i], nq);
                mbar_init(&pv_free[t * NPB + i], 1);
            }
            mbar_init(&o_ready[t], 1);
        }
        mbar_init(mma_done, 2);
        mbar_init(never, 1);
        // a CTA started after another one gave up a wait does no work (a systematic failure ends in one timeout)
        *abort_flag = *(volatile int *) p.status != ST_OK;
        fence_mbar_init();
    }
    __syncthreads();
    if (*abort_flag) return;   // uniform: before TMEM is allocated
    if (warp == 1) {   // TMEM: per tile S, two P buffers and O; one tile: a second S
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // NT == 2: 16 warps launched with 128 registers each; every warpgroup's branch starts by resizing its share:
    // control 128 (TMA and the MMA issuers), softmax 2 x 152, dequant 80 (128 x (128 + 152 + 152 + 80) = 65,536 = the
    // launched total): the split at which no role spills

    auto wait = [&](uint64_t *b, uint32_t parity) -> bool {
        if (!ok) return false;
        if (!mbar_wait_bounded(b, parity, tmo, abort_flag)) {
            ok = false;
            *abort_flag = 1;
            atomicCAS(p.status, ST_OK, ST_TIMEOUT_FULL);
        }
        return ok;
    };

    if (warp < 4) {
      // 16 warps launched with 128 registers each at NT = 1 and 2; each warpgroup resizes its share (NT = 1, 64-key
      // blocks: control 160, softmax 168, two dequant warpgroups 88; 128-key blocks: control 128, softmax 200 (the 128
      // scores of a row), dequant 88: 128 x (160 + 168 + 88 + 88) or 128 x (128 + 200 + 88 + 88) = 64,512 <= 65,536)
      if constexpr (NT == 1 && B == 64) asm volatile("setmaxnreg.inc.sync.aligned.u32 160;");
      if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            if constexpr (!QT) {
                const int qrow = (int) (((uint64_t) job.set * p.nkv + h) * p.rows + row0);
                mbar_arrive_expect_tx(q_full, NT * BM * D * 2);
                for (int t = 0; t < NT; t++)
                    for (int c = 0; c < D / 64; c++)
                        tma_2d(smem + L::Q + t * BM * D * 2 + c * BM * 128, &tq, c * 64, qrow + t * BM, q_full);
            }
            const CUtensorMap *km = p.kv_maps + 2 * job.seg, *vm = km + 1;
            uint32_t issued = 0;
            for (uint32_t j = 0; j < nblk; j++) {
                const uint32_t st = j % NRS;
                if (j >= NRS && !wait(&raw_empty[st], ((j / NRS) - 1) & 1)) break;
                mbar_arrive_expect_tx(&raw_full[st], 2 * B * RAWB);
                uint8_t *dst = smem + L::RAW + st * L::RAW_STAGE;
#pragma unroll
                for (int c = 0; c < B / BN; c++) {   // the tensor maps' boxes hold 64 keys
                    const int key = (int) (job.key0 + j * B) + c * BN;
                    tma_2d(dst + c * BN * RAWB, km, hx / 2, key, &raw_full[st]);
                    tma_2d(dst + (B + c * BN) * RAWB, vm, hx / 2, key, &raw_full[st]);
                }
                issued = j + 1;
            }
            // on an abort, every issued copy lands before the CTA exits
            if (!ok) {
                const uint64_t drain = tmo > dec::DRAIN_NS ? tmo : dec::DRAIN_NS;
                if (!QT && !mbar_wait_bounded(q_full, 0, drain, nullptr)) atomicCAS(p.status, ST_OK, ST_TIMEOUT_DRAIN);
                const uint32_t first = issued > NRS ? issued - NRS : 0;
                for (uint32_t j = first; j < issued; j++)
                    if (!mbar_wait_bounded(&raw_full[j % NRS], (j / NRS) & 1, drain, nullptr))
                        atomicCAS(p.status, ST_OK, ST_TIMEOUT_DRAIN);
            }
        }
      } else if (warp == 1 || warp == 2) {
        // ------------------------------------------------ MMA issuers: warp 1 the S = Q K^T MMAs, warp 2 the P.V ones.
        // Two issuing threads (on two SM sub-partitions) keep the issue of one kind from waiting behind the other;
        // each commit tracks its own thread's MMAs, and the softmax orders the two through s_full / p_full / pv_free.
        // Operand descriptors are built once: their high word (LBO, SBO, version, swizzle) is fixed per operand and an
        // operand's start address advances by adding (byte offset >> 4) to the 14-bit start field (every address
        // stays below 256 KB, so the field cannot carry).
        if (lane == 0 && warp == 1) {
            const uint64_t dq0 = sdesc(sbase + L::Q, 16, 1024), dk0 = sdesc(sbase + L::K, 16, 1024);
            if (wait(q_full, 0)) {
                for (uint32_t j = 0; j < nblk && ok; j++) {
                    const uint32_t b = j % KVB;
                    if (!wait(&k_full[b], (j / KVB) & 1)) break;
                    const uint64_t dk = dk0 + b * (uint32_t) (B * D * 2 / 16);
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                        const uint32_t sb = t * NSB + j % NSB;   // the block's S buffer
                        if (j >= NSB && !wait(&s_empty[sb], ((j / NSB) - 1) & 1)) break;
                        tc_fence_after();
                        const uint32_t d = tmem + t * 256 + (j % NSB) * 256;
                        const uint64_t dq = dq0 + (uint32_t) (t * BM * D * 2 / 16);
#pragma unroll
                        for (int kk = 0; kk < D / 16; kk++) {
                            const uint64_t bk = dk + (uint32_t) (((kk / 4) * B * 128 + (kk % 4) * 32) / 16);
                            if constexpr (QT)   // A = Q from tensor memory: 8 columns (16 f16) per k-step
                                tc_mma_ts(d, tmem + t * 256 + T_Q + kk * 8, bk, IDESC_S, kk > 0 ? 1u : 0u);
                            else
                                tc_mma(d, dq + (uint32_t) (((kk / 4) * BM * 128 + (kk % 4) * 32) / 16), bk, IDESC_S,
                                       kk > 0 ? 1u : 0u);
                        }
                        tc_commit(&s_full[sb]);
                    }
                    if (!ok) break;
                    tc_commit(&k_free[b]);
                }
            }
        } else if (lane == 0) {
            const uint64_t dv0 = sdesc(sbase + L::V, B * 128, 1024);
            for (uint32_t jj = 0; jj < nblk && ok; jj++) {
                const uint32_t b = jj % KVB;   // V buffer
                if (!wait(&v_full[b], (jj / KVB) & 1)) break;
                const uint64_t dv = dv0 + b * (uint32_t) (B * D * 2 / 16);
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    const uint32_t pb = jj % NPB;   // P buffer
                    if (!wait(&p_full[t * NPB + pb], (jj / NPB) & 1)) break;
                    tc_fence_after();
                    const uint32_t d = tmem + t * 256 + T_O;
                    const uint32_t pa = tmem + t * 256 + p_col(pb);   // P buffer pb (f16, two keys per column)
#pragma unroll
                    for (int ks = 0; ks < B / 16; ks++)
                        tc_mma_ts(d, pa + ks * 8, dv + (uint32_t) (ks * 2048 / 16), IDESC_PV, (jj > 0 || ks > 0) ? 1u : 0u);
                    tc_commit(&pv_free[t * NPB + pb]);   // P buffer pb and O (through this block) are settled
                    if (jj + 1 == nblk) tc_commit(&o_ready[t]);
                }
                if (!ok) break;
                tc_commit(&v_free[b]);
            }
        }
        if (lane == 0) {
            // TMEM must not be released under MMAs still running (they complete on their own; bounded wait): both
            // issuers commit to mma_done (count 2) and wait for both
            tc_commit(mma_done);
            const uint64_t drain = tmo > dec::DRAIN_NS ? tmo : dec::DRAIN_NS;
            if (!mbar_wait_bounded(mma_done, 0, drain, nullptr)) atomicCAS(p.status, ST_OK, ST_TIMEOUT_DRAIN);
        }
      }   // warp 3: idle
    } else if (warp < (uint32_t) DQ0) {
        // ------------------------------------------------ softmax warpgroup of tile t
        if constexpr (NT == 2) asm volatile("setmaxnreg.inc.sync.aligned.u32 152;");
        else if constexpr (B == 128) asm volatile("setmaxnreg.inc.sync.aligned.u32 200;");
        else asm volatile("setmaxnreg.inc.sync.aligned.u32 168;");
        if (p.stall) wait(never, 0);                       // runs out: records the timeout, every role unwinds
        const int t = (int) (warp - SM0) / 4;
        const uint32_t wq = warp % 4;                      // TMEM lane quarter of this warp
        const uint32_t r = wq * 32 + lane;                 // row of the tile = TMEM lane
        const uint32_t tl = tmem + ((wq * 32) << 16) + t * 256;
        // a warp whose 32 rows are all past the call's rows (a partly filled tile; NT = 1 only) sits the blocks out: the
        // S, P and Q barriers count only the warps with a real row, its rows' O is never written and MMA rows are
        // independent, so its S, P and Q may stay as they are. (It must not arrive at all: a warp that does no work can
        // run ahead of the real warps, and its arrival for a later block would complete an earlier block's phase.)
        const bool pad = NT == 1 && row0 + t * BM + wq * 32 >= p.rows;
        // Q in tensor memory: each warp with a real row writes its lanes' Q rows (rows past the call's rows as zeros)
        // into the Q columns, then arrives on q_full, which the S issuer waits for
        if constexpr (QT) {
            if (!pad && ok) {
                const uint32_t row = row0 + r;
                const uint4 *src =
                    reinterpret_cast<const uint4 *>(p.Qs + (((uint64_t) job.set * p.nkv + h) * p.rows + row) * D);
#pragma unroll
                for (int c = 0; c < D / 64; c++) {   // 64 dims (32 columns) at a time
                    uint32_t qv[32];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const uint4 v = row < p.rows ? __ldg(src + 8 * c + i) : make_uint4(0u, 0u, 0u, 0u);
                        qv[4 * i] = v.x; qv[4 * i + 1] = v.y; qv[4 * i + 2] = v.z; qv[4 * i + 3] = v.w;
                    }
                    tmem_st32u(tl + T_Q + 32 * c, qv);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(q_full);
            }
        }
        float m_used = -INFINITY, l = 0.f;
        float m_row = -INFINITY;   // the row's exact maximum (log2 units); O and l are reported against it
        for (uint32_t j = 0; j < nblk && !pad; j++) {
            const uint32_t b = j % NPB;                    // the block's P buffer
            const uint32_t sb = t * NSB + j % NSB;         // the block's S buffer
            if (!wait(&s_full[sb], (j / NSB) & 1)) break;
            tc_fence_after();
            const uint32_t ts = tl + (j % NSB) * 256;
            float s[B];   // the row's B scores stay in registers, so S is free as soon as it is read
            {
                float a[B / 32][32];
#pragma unroll
                for (int c = 0; c < B / 32; c++) tmem_ld32(ts + 32 * c, a[c]);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < B / 32; c++)
#pragma unroll
                    for (int i = 0; i < 32; i++) s[32 * c + i] = a[c][i];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[sb]);
            const int nvalid = (int) (job.nk - j * B);
            if (nvalid < B) {
#pragma unroll
                for (int i = 0; i < B; i++)
                    if (i >= nvalid) s[i] = -INFINITY;
            }
            float mx = s[0];
#pragma unroll
            for (int i = 1; i + 1 < B; i += 2) mx = max3(mx, s[i], s[i + 1]);
            mx = fmaxf(mx, s[B - 1]);
            mx *= LOG2E;
            m_row = fmaxf(m_row, mx);
            float alpha = 1.f;
            bool rescale = false;
            if (j == 0) m_used = mx;
            else if (mx > m_used + 8.f) {
                alpha = ex2(m_used - mx);
                m_used = mx;
                rescale = true;
            }
            // p = 2^(s*log2e - m): scale-and-shift and the row sum on fp32 pairs (fma/add .f32x2)
            const uint64_t l2e2 = pack_f2(LOG2E, LOG2E), nm2 = pack_f2(-m_used, -m_used);
            uint64_t acc = pack_f2(0.f, 0.f);
            uint32_t ph[B / 2];
#pragma unroll
            for (int i = 0; i < B / 2; i++) {
                float t0, t1;
                unpack_f2(fma_f2(pack_f2(s[2 * i], s[2 * i + 1]), l2e2, nm2), t0, t1);
                const float p0 = ex2(t0), p1 = ex2(t1);
                acc = add_f2(acc, pack_f2(p0, p1));
                ph[i] = pack_h2(p0, p1);
            }
            float sum_a, sum_b;
            unpack_f2(acc, sum_a, sum_b);
            l = fmaf(l, alpha, sum_a + sum_b);
            // O is rescaled (rarely: the lazy max moved) once P.V of block j-1 has completed; P buffer b is free once
            // P.V of block j-NPB (its last reader) has. Each buffer's barrier completes once per P.V on that buffer,
            // and P.V of block j cannot start before this P is written, so each wait names exactly one completion.
            if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
                if (!wait(&pv_free[t * NPB + (j - 1) % NPB], ((j - 1) / NPB) & 1)) break;
                tc_fence_after();
#pragma unroll
                for (int q = 0; q < D / 32; q++) {
                    float o[32];
                    tmem_ld32(tl + T_O + q * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < 32; x++) o[x] *= alpha;
                    tmem_st32(tl + T_O + q * 32, o);
                }
                tmem_wait_st();
            }
            if (j >= NPB && !wait(&pv_free[t * NPB + b], ((j / NPB) - 1) & 1)) break;
            // P, two keys per column, into P buffer b (32 columns at a time)
#pragma unroll
            for (int hq = 0; hq < B / 64; hq++)
                tmem_st32u(tl + p_col(b) + 32 * hq, *reinterpret_cast<const uint32_t(*)[32]>(ph + 32 * hq));
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t * NPB + b]);
        }
        // final: O from TMEM to the slot partial, moved from the lazy reference max m_used to the row's exact maximum
        // (m = max_j s_j, as sme_attn_partial reports it): one factor 2^(m_used - m_row) in (2^-8, 1] on O and l
        if (ok && !pad && nblk > 0 && wait(&o_ready[t], 0)) {
            tc_fence_after();
            const uint32_t row = row0 + t * BM + r;
            const uint64_t orow = ((uint64_t) job.slot * p.nkv + h) * p.rows + row;
            const float fix = m_row > -INFINITY ? ex2(m_used - m_row) : 1.f;
#pragma unroll
            for (int q = 0; q < D / 32; q++) {
                float o[32];
                tmem_ld32(tl + T_O + q * 32, o);
                tmem_wait_ld();
                if (row < p.rows) {
                    float4 *dst = reinterpret_cast<float4 *>(p.Op + orow * D + q * 32);
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        dst[i] = make_float4(o[4 * i] * fix, o[4 * i + 1] * fix, o[4 * i + 2] * fix, o[4 * i + 3] * fix);
                }
            }
            if (row < p.rows) {
                p.Mp[orow] = l > 0.f ? m_row * (1.0f / LOG2E) : -INFINITY;
                p.Lp[orow] = l * fix;
            }
        }
    } else {
        // ------------------------------------------------ dequantisers: warp dw owns quant blocks dw % 4 (+ 4 at
        // D = 256) of every key (4 warps: both 32-key halves of each 64 keys; 8 warps, NT = 1: key half dw / 4 of each
        // 64 keys)
        if (NT == 2) asm volatile("setmaxnreg.dec.sync.aligned.u32 80;");
        else asm volatile("setmaxnreg.dec.sync.aligned.u32 88;");
        const uint32_t dw = warp - DQ0;
        for (uint32_t j = 0; j < nblk; j++) {
            const uint32_t st = j % NRS, b = j % KVB;
            if (!wait(&raw_full[st], (j / NRS) & 1)) break;
            const uint32_t raw = sbase + L::RAW + st * L::RAW_STAGE;
#pragma unroll
            for (int kv = 0; kv < 2; kv++) {
                if (j >= KVB && !wait(kv == 0 ? &k_free[b] : &v_free[b], ((j / KVB) - 1) & 1)) break;
                const uint32_t src = raw + kv * B * RAWB;
                // items: 64-key chunk kc of the block, key half (8 warps) or pass (4 warps), quant block of the warp
#pragma unroll
                for (int it = 0; it < (B / 64) * (8 / NDQ) * (D / 128); it++) {
                    const int pass = it % (8 / NDQ), kc = it / (8 / NDQ) % (B / 64);
                    const uint32_t qblk = dw % 4 + 4 * (uint32_t) (it / ((8 / NDQ) * (B / 64)));
                    const uint32_t bo = hoff + GB * qblk;               // block start inside the raw window row
                    const uint32_t w16 = bo & ~15u;                     // 16-byte aligned start of the words covering it
                    const uint32_t ds = bo + 2;                         // first data byte
                    const uint32_t w0 = (ds - w16) / 4, shift = 8 * (ds % 4);
                    // atom column of this block's d's
                    const uint32_t dst = sbase + (kv == 0 ? L::K : L::V) + b * B * D * 2 + (qblk / 2) * B * 128;
                    const uint32_t key = 64 * (uint32_t) kc + (NDQ == 8 ? dw / 4 : (uint32_t) pass) * 32 + lane;
                    const uint32_t rb = src + key * RAWB;
                    const uint32_t s2 = lds16(rb + bo);
                    const uint32_t sc2 = s2 | (s2 << 16);
                    uint32_t W[12];
                    // q8_0: the block's 34 bytes lie within 3 aligned 16-byte chunks; q4_0: 18 bytes within 2
#pragma unroll
                    for (int i = 0; i < (QUANT == 1 ? 3 : 2); i++)
                        lds128(rb + w16 + 16 * i, W[4 * i], W[4 * i + 1], W[4 * i + 2], W[4 * i + 3]);
                    if (QUANT != 1) W[8] = W[9] = W[10] = W[11] = 0u;
                    const uint32_t kbase = dst + (key / 8) * 1024 + (key % 8) * 128;
                    if (QUANT == 1) {
                        uint32_t A[8];
                        switch (w0) {   // uniform across the warp
#define PA_ALIGN8(W0)                                                                        \
    case W0:                                                                                 \
        _Pragma("unroll") for (int i = 0; i < 8; i++) A[i] = __funnelshift_r(W[W0 + i], W[(W0 + i + 1 < 12) ? W0 + i + 1 : 11], shift); \
        break;
                            PA_ALIGN8(0) PA_ALIGN8(1) PA_ALIGN8(2) PA_ALIGN8(3) default: PA_ALIGN8(4)
#undef PA_ALIGN8
                        }
#pragma unroll
                        for (int cc = 0; cc < 4; cc++) {
                            uint32_t h0, h1, h2, h3;
                            dec::q8_word(A[2 * cc], sc2, h0, h1);
                            dec::q8_word(A[2 * cc + 1], sc2, h2, h3);
                            const uint32_t c = 4 * (qblk % 2) + cc;
                            sts128(kbase + ((c ^ (key % 8)) * 16), h0, h1, h2, h3);
                        }
                    } else {
                        uint32_t AW[4];
                        switch (w0) {
#define PA_ALIGN4(W0)                                                                        \
    case W0:                                                                                 \
        _Pragma("unroll") for (int i = 0; i < 4; i++) AW[i] = __funnelshift_r(W[W0 + i], W[W0 + i + 1], shift); \
        break;
                            PA_ALIGN4(0) PA_ALIGN4(1) PA_ALIGN4(2) PA_ALIGN4(3) default: PA_ALIGN4(4)
#undef PA_ALIGN4
                        }
                        // byte i: element i (low nibble), element i + 16 (high nibble)
                        uint32_t lo[8], hi[8];   // f16x2 of elements (2i, 2i+1) and (16+2i, 17+2i)
                        const uint32_t m = 0x000F000Fu, magic = 0x64006400u, off8 = 0x64086408u;
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const uint32_t y = prmt(AW[i], AW[i], 0x3120u);   // bytes (x0, x2, x1, x3)
                            lo[2 * i] = hmul2(hsub2(and_or(y, m, magic), off8), sc2);
                            lo[2 * i + 1] = hmul2(hsub2(and_or(y >> 8, m, magic), off8), sc2);
                            hi[2 * i] = hmul2(hsub2(and_or(y >> 4, m, magic), off8), sc2);
                            hi[2 * i + 1] = hmul2(hsub2(and_or(y >> 12, m, magic), off8), sc2);
                        }
                        const uint32_t c0 = 4 * (qblk % 2);
                        sts128(kbase + (((c0 + 0) ^ (key % 8)) * 16), lo[0], lo[1], lo[2], lo[3]);
                        sts128(kbase + (((c0 + 1) ^ (key % 8)) * 16), lo[4], lo[5], lo[6], lo[7]);
                        sts128(kbase + (((c0 + 2) ^ (key % 8)) * 16), hi[0], hi[1], hi[2], hi[3]);
                        sts128(kbase + (((c0 + 3) ^ (key % 8)) * 16), hi[4], hi[5], hi[6], hi[7]);
                    }
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(kv == 0 ? &k_full[b] : &v_full[b]);
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[st]);
        }
    }

    // every role ends here (no return after the TMEM allocation); the MMA thread has waited for its MMAs
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
    }
}

}  // namespace pre
}  // namespace pa
