// pa_prefill_pair.cuh - the tcgen05 prefill kernel on CTA pairs: each MMA is a 2-SM MMA (cta_group::2, M = 256) that
// reads A (Q rows, or P from tensor memory) from both CTAs and B split by N across them, so each SM dequantises half
// of every K/V block and one thread issues the MMAs of both SMs.
//
// Reference semantics: pa_attn_big (phone-attn/pa-metal.mm:379-487), as in pa_prefill.cuh: rows of all groups of one
// KV head packed back to back, K/V dequantised to f16, S = Qs.K^T and O += P.V with fp32 accumulation, online softmax
// over the valid keys, one unnormalised (O, m, l) per chunk of keys. Head dim D = 128 (NT = 1 or 2 pair tiles) or 256
// (the reference server's wire geometry, phone-attn/phone-attn.h:79; NT = 1: TMEM holds NT x (64 + 64 + D) columns).
//
// One cluster of 2 CTAs = one chunk of keys of one segment x one KV head x NT pair tiles of 256 query rows; CTA r of
// the pair holds rows [128 r, 128 r + 128) of each pair tile (its TMEM lanes), and of each 64-key block
//   K: keys [32 r, 32 r + 32), all D dims (the N half of B for S = Q K^T, N = 64 keys)
//   V: all 64 keys, dims [D r / 2, D (r + 1) / 2) (the N half of B for O += P V, N = D dims)
// Warp roles in each CTA (as in pa_prefill.cuh):
//   warp 0             TMA: its Q tiles once, then per block its raw K rows (32 keys) and V rows (64 keys)
//   warps 1, 2, 3      warp 1 allocates TMEM (both CTAs, cta_group::2). In CTA 0 one thread of warp 1 issues the S
//                      MMAs of pair tile 0, one of warp 3 those of tile 1 and one of warp 2 the P.V MMAs, for both
//                      CTAs; their commits arrive on the barrier at the same offset in both CTAs (multicast commit).
//                      In CTA 1, warp 1 tells CTA 0 its Q is in place.
//   warps 4 .. 4+4NT   softmax of pair tile t for this CTA's 128 rows
//   last 4 (D = 128) or dequantise this CTA's halves of each K and V block
//   8 (D = 256) warps
// Operand-ready and buffer-free arrivals of both CTAs' dequant and softmax warps go to CTA 0's barriers over
// distributed shared memory (8 arrivals: 4 warps x 2 CTAs). Each is preceded by the wait that completes what it
// publishes (shared stores: fence.proxy.async; TMEM: tcgen05.wait::st / ::ld), and is a remote arrive with the default
// (CTA-scope) release, as CUTLASS's cluster barriers arrive on a peer: a cluster-scope release arrive measured
// 500-775 ns under this kernel's load against ~80 ns, and a relay thread issuing those serialised the pipeline. No TMA
// copy multicasts.
// All waits are bounded; both CTAs reach the final cluster barrier on every path, so neither exits while the other
// can still reach its shared memory, and TMEM is released by both.
#pragma once
#include "pa_prefill.cuh"

namespace pa {
namespace pre {

// ---------------------------------------------------------------- cluster helpers
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the shared::cluster address of this CTA's shared address `a` in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa(uint32_t a, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t cl_addr) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cl_addr) : "memory");
    return v;
}
// arrive on an mbarrier of any CTA of the cluster (default semantics: release, CTA scope)
__device__ __forceinline__ void mbar_arrive_cl(uint32_t cl_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}
// wait (bounded) on a barrier that CTAs of the cluster arrive on (acquire at cluster scope)
__device__ __forceinline__ bool mbar_try_wait_cl(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded_cl(uint64_t *bar, uint32_t parity, uint64_t timeout_ns,
                                                     const volatile int *abort) {
    if (mbar_try_wait_cl(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; it++) {
        if (mbar_try_wait_cl(bar, parity)) return true;
        if ((it & 63) == 63) {
            if (abort != nullptr && *abort) return false;
            if (globaltimer_ns() - t0 > timeout_ns) return false;
        }
    }
}

// 2-SM MMAs (issued by CTA 0 of the pair; descriptors and TMEM addresses name the same offsets in both CTAs)
__device__ __forceinline__ void tc2_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tc2_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc));
}
// completion of this thread's MMAs arrives once on the mbarrier at this offset in both CTAs of the pair
__device__ __forceinline__ void tc2_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "h"((uint16_t) 3)
                 : "memory");
}

// shared-memory map of a CTA of the pair (operand tiles 1024-aligned); D = head dim (128 or 256)
template <int QUANT, int NT, int D>
struct PairSmem {
    static constexpr int RAWB = raw_row_bytes(QUANT, D);
    static constexpr int KH = BN / 2;                              // keys of K per CTA per block
    static constexpr int KVB = D == 128 ? 4 : 2;                   // dequantised K and V buffers (a ring)
    static constexpr int TS = 128 + D;                             // TMEM columns per pair tile: S 64, P 2 x 32, O D
    static constexpr int TMEM_COLS = NT * TS <= 256 ? 256 : 512;   // allocation: a power of 2
    static constexpr int Q = 0;                                   // NT x [D/64 atom cols][128 rows][128 B]
    static constexpr int K_BUF = (D / 64) * KH * 128;              // [D/64 atom cols][32 keys][128 B]
    static constexpr int V_BUF = (D / 128) * BN * 128;             // [D/128 atom cols][64 keys][128 B] (this CTA's D/2 dims)
    static constexpr int K = Q + NT * BM * D * 2;                  // KVB K buffers
    static constexpr int V = K + KVB * K_BUF;                      // KVB V buffers
    static constexpr int RAW = V + KVB * V_BUF;                    // NS x (K rows [32][RAWB], V rows [64][RAWB])
    static constexpr int RAW_V = KH * RAWB;                        // V rows' offset inside a stage
    static constexpr int RAW_STAGE = ((KH + BN) * RAWB + 1023) / 1024 * 1024;
    static constexpr int BAR = RAW + NS * RAW_STAGE;
    static constexpr int N_BAR = 2 + 2 * NS + 4 * KVB + 7 * NT + 1 + 1;
    static constexpr int TOTAL = BAR + N_BAR * 8 + 32;
};

// dequant warps per CTA: 4 at D = 128; 8 at D = 256 (one pair tile per CTA, and twice the dims per key)
__host__ __device__ constexpr int pair_dq_warps(int d) { return d == 128 ? 4 : 8; }
// A dequant lane's (key, quant block) item: pass ps of operand kv (0 = K, 1 = V) for dequant warp dw (of NDQ) and lane
// `lane` of CTA cr. ql: block within this CTA's tile, qb: block of the head, key: key row in the raw stage.
//   K: 32 keys x D/32 blocks; NDQ = 4: pass ps, warp dw: block dw + 4 ps of key `lane`; NDQ = 8: block dw
//   V: 64 keys x D/64 blocks (this CTA's dims: blocks cr D/64 ..); NDQ = 4: block cr D/64 + (dw & 1) + 2 ps of key
//      32 (dw >> 1) + lane; NDQ = 8: block cr D/64 + (dw & 3) of key 32 (dw >> 2) + lane
template <int D, int NDQ>
__host__ __device__ __forceinline__ void dq_item(int kv, int ps, uint32_t dw, uint32_t lane, uint32_t cr, uint32_t &ql,
                                                 uint32_t &qb, uint32_t &key) {
    if (NDQ == 4) {
        ql = kv == 0 ? dw + 4 * (uint32_t) ps : (dw & 1) + 2 * (uint32_t) ps;
        key = kv == 0 ? lane : (dw >> 1) * 32 + lane;
    } else {
        ql = kv == 0 ? dw : (dw & 3);
        key = kv == 0 ? lane : (dw >> 2) * 32 + lane;
    }
    qb = kv == 0 ? ql : cr * (D / 64) + ql;
}
// Where an item goes in its operand buffer: K [D/64 atom cols][32 keys][128 B], V [D/128 atom cols][64 keys][128 B],
// an atom column = 64 dims = 2 blocks. dq_row: byte offset of the key's 128-byte row in the item's atom column;
// dq_chunk: offset of 16-byte chunk cc (8 f16) of the item in that row, chunk 4 (ql % 2) + cc swizzled by key % 8 (the
// UMMA 128-byte swizzle)
__host__ __device__ __forceinline__ uint32_t dq_row(int kv, uint32_t ql, uint32_t key) {
    return (ql / 2) * (kv == 0 ? BN / 2 : BN) * 128 + (key / 8) * 1024 + (key % 8) * 128;
}
__host__ __device__ __forceinline__ uint32_t dq_chunk(uint32_t ql, uint32_t key, uint32_t cc) {
    return ((4 * (ql % 2) + cc) ^ (key % 8)) * 16;
}

template <int QUANT, int NT, int D>
__global__ void __launch_bounds__(32 * (4 + 4 * NT + pair_dq_warps(D)), 1) prefill_pair_kernel(const __grid_constant__ CUtensorMap tq,
                                                                            const Params p) {
    using L = PairSmem<QUANT, NT, D>;
    static_assert((D == 128 && (NT == 1 || NT == 2)) || (D == 256 && NT == 1), "TMEM holds NT x (128 + D) columns");
    constexpr int RAWB = L::RAWB, KH = L::KH, KVB = L::KVB, TS = L::TS;
    constexpr int GB = dec::q_group_bytes(QUANT);
    constexpr uint32_t IDESC_S = idesc_f16(2 * BM, BN, 0);
    constexpr uint32_t IDESC_PV = idesc_f16(2 * BM, D, 1);
    constexpr int SM0 = 4, DQ0 = 4 + 4 * NT;   // first softmax warp, first dequant warp
    constexpr int NDQ = pair_dq_warps(D), NPASS = (D / 128) * 4 / NDQ;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const uint32_t sbase = smem_u32(smem);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L::BAR);
    uint64_t *q_full = bar;                    // this CTA's Q tiles landed
    uint64_t *q_pair = bar + 1;                // (CTA 0) CTA 1's Q tiles landed
    uint64_t *raw_full = bar + 2, *raw_empty = raw_full + NS;
    uint64_t *k_full = raw_empty + NS, *k_free = k_full + KVB, *v_full = k_free + KVB, *v_free = v_full + KVB;
    uint64_t *s_full = v_free + KVB;           // [NT]
    uint64_t *s_empty = s_full + NT;           // [NT] (CTA 0: both CTAs' softmax read S)
    uint64_t *p_full = s_empty + NT;           // [NT][2] (CTA 0: both CTAs' P of the block in buffer b)
    uint64_t *pv_free = p_full + 2 * NT;       // [NT][2]
    uint64_t *o_ready = pv_free + 2 * NT;      // [NT]
    uint64_t *mma_done = o_ready + NT;         // both issuers' MMAs completed
    uint64_t *never = mma_done + 1;            // completed by nobody: the stall test hook waits on it
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + L::N_BAR);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const uint32_t cr = cluster_rank();
    // cluster order (a 1-D grid of CTA pairs): row-tile group fastest, then KV head, then job, so the clusters that read
    // the same K/V blocks (all row groups and heads of one chunk of keys) run at the same time and share them through L2
    const uint32_t cid = blockIdx.x / 2;
    const uint32_t rt = cid % p.n_rt, h = (cid / p.n_rt) % p.nkv;
    const dec::Job job = p.jobs[cid / (p.n_rt * p.nkv)];
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t nblk = (job.nk + BN - 1) / BN;
    const uint32_t hbyte = h * (uint32_t) p.hb;
    const int hx = (int) (hbyte & ~15u);
    const uint32_t hoff = hbyte & 15u;
    const uint32_t row0 = rt * NT * 2 * BM;       // first query row of this pair (within the head)
    const uint64_t tmo = p.timeout_ns;
    bool ok = true;
    // CTA 0's barrier at the same offset as `b`, as a shared::cluster address (arrivals of both CTAs go there)
    auto lead = [&](uint64_t *b) -> uint32_t { return mapa(smem_u32(b), 0); };

    if (threadIdx.x == 0) {
        // operand-ready barriers of CTA 0: NDQ dequant warps of each CTA; buffer-free (S read, P written): 4 softmax
        // warps of each CTA
        constexpr uint32_t npair = 8, nopnd = 2 * NDQ;
        mbar_init(q_full, 1);
        mbar_init(q_pair, 1);
        for (int s = 0; s < NS; s++) { mbar_init(&raw_full[s], 1); mbar_init(&raw_empty[s], NDQ); }
        for (int b = 0; b < KVB; b++) {
            mbar_init(&k_full[b], nopnd); mbar_init(&k_free[b], NT); mbar_init(&v_full[b], nopnd); mbar_init(&v_free[b], 1);
        }
        for (int t = 0; t < NT; t++) {
            mbar_init(&s_full[t], 1);
            mbar_init(&s_empty[t], npair);
            mbar_init(&p_full[2 * t], npair);
            mbar_init(&p_full[2 * t + 1], npair);
            mbar_init(&pv_free[2 * t], 1);
            mbar_init(&pv_free[2 * t + 1], 1);
            mbar_init(&o_ready[t], 1);
        }
        mbar_init(mma_done, 1 + NT);
        mbar_init(never, 1);
        *abort_flag = cr == 0 && *(volatile int *) p.status != ST_OK;
        fence_mbar_init();
    }
    // both CTAs' barriers initialised before any arrival crosses; the pair takes CTA 0's decision to skip the work
    // of a call that already failed (uniform, before TMEM is allocated), and neither exits before both have read it
    cluster_sync();
    const uint32_t skip = ld_cluster_u32(mapa(smem_u32((const void *) abort_flag), 0));
    cluster_sync();
    if (skip) return;
    if (warp == 1) {   // TMEM: per pair tile S 64 + P 2 x 32 + O D columns, the same columns in both CTAs
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(L::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto wait = [&](uint64_t *b, uint32_t parity) -> bool {
        if (!ok) return false;
        if (!mbar_wait_bounded(b, parity, tmo, abort_flag)) {
            ok = false;
            *abort_flag = 1;
            atomicCAS(p.status, ST_OK, ST_TIMEOUT_FULL);
        }
        return ok;
    };
    auto wait_cl = [&](uint64_t *b, uint32_t parity) -> bool {
        if (!ok) return false;
        if (!mbar_wait_bounded_cl(b, parity, tmo, abort_flag)) {
            ok = false;
            *abort_flag = 1;
            atomicCAS(p.status, ST_OK, ST_TIMEOUT_FULL);
        }
        return ok;
    };

    if (warp < 4) {
      // NT = 2 (D = 128) and D = 256 launch 16 warps with 128 registers each, and every warpgroup resizes its share:
      // NT = 2: control 128, softmax 2 x 152, dequant 80; D = 256: control 160, softmax 168, dequant 2 x 88
      if (NT == 2) asm volatile("setmaxnreg.dec.sync.aligned.u32 128;");
      if (D == 256) asm volatile("setmaxnreg.inc.sync.aligned.u32 160;");
      if (warp == 0) {
        // ------------------------------------------------ TMA producer (each CTA its own operands)
        if (lane == 0) {
            const int qrow = (int) (((uint64_t) job.set * p.nkv + h) * p.rows + row0 + cr * BM);
            mbar_arrive_expect_tx(q_full, NT * BM * D * 2);
            for (int t = 0; t < NT; t++)
                for (int c = 0; c < D / 64; c++)
                    tma_2d(smem + L::Q + t * BM * D * 2 + c * BM * 128, &tq, c * 64, qrow + t * 2 * BM, q_full);
            const CUtensorMap *km = p.kv_maps + 2 * job.seg, *vm = km + 1;
            uint32_t issued = 0;
            for (uint32_t j = 0; j < nblk; j++) {
                const uint32_t st = j % NS;
                if (j >= NS && !wait(&raw_empty[st], ((j / NS) - 1) & 1)) break;
                mbar_arrive_expect_tx(&raw_full[st], (KH + BN) * RAWB);
                uint8_t *dst = smem + L::RAW + st * L::RAW_STAGE;
                tma_2d(dst, km, hx / 2, (int) (job.key0 + j * BN + cr * KH), &raw_full[st]);
                tma_2d(dst + L::RAW_V, vm, hx / 2, (int) (job.key0 + j * BN), &raw_full[st]);
                issued = j + 1;
            }
            if (!ok) {
                const uint64_t drain = tmo > dec::DRAIN_NS ? tmo : dec::DRAIN_NS;
                if (!mbar_wait_bounded(q_full, 0, drain, nullptr)) atomicCAS(p.status, ST_OK, ST_TIMEOUT_DRAIN);
                const uint32_t first = issued > NS ? issued - NS : 0;
                for (uint32_t j = first; j < issued; j++)
                    if (!mbar_wait_bounded(&raw_full[j % NS], (j / NS) & 1, drain, nullptr))
                        atomicCAS(p.status, ST_OK, ST_TIMEOUT_DRAIN);
            }
        }
      } else if (warp == 1 || warp == 2 || (warp == 3 && NT == 2)) {
        if (cr == 0 && lane == 0 && warp != 2) {
            // ------------------------------------------------ S = Q K^T issuers (M = 256 over the pair, N = 64 keys):
            // warp 1 for pair tile 0, warp 3 for tile 1 (an MMA of this shape holds its issuing thread ~100 cycles, so
            // one thread per tile doubles the issue rate)
            const int t = warp == 1 ? 0 : 1;
            const uint64_t dq = sdesc(sbase + L::Q + t * BM * D * 2, 16, 1024), dk0 = sdesc(sbase + L::K, 16, 1024);
            const uint32_t d = tmem + t * TS;
            if (wait(q_full, 0) && wait_cl(q_pair, 0)) {
                for (uint32_t j = 0; j < nblk && ok; j++) {
                    const uint32_t b = j % KVB;
                    if (!wait_cl(&k_full[b], (j / KVB) & 1)) break;
                    if (j >= 1 && !wait_cl(&s_empty[t], (j - 1) & 1)) break;
                    tc_fence_after();
                    const uint64_t dk = dk0 + b * (uint32_t) (L::K_BUF / 16);
#pragma unroll
                    for (int kk = 0; kk < D / 16; kk++)
                        tc2_mma(d, dq + (uint32_t) (((kk / 4) * BM * 128 + (kk % 4) * 32) / 16),
                                dk + (uint32_t) (((kk / 4) * KH * 128 + (kk % 4) * 32) / 16), IDESC_S, kk > 0 ? 1u : 0u);
                    tc2_commit(&s_full[t]);
                    tc2_commit(&k_free[b]);   // count NT: every tile's S MMAs of the block have read K buffer b
                }
            }
        } else if (cr == 0 && lane == 0) {
            // ------------------------------------------------ O += P V issuer (M = 256, N = D dims, A = P in TMEM; B:
            // this CTA's D/2 dims, D/128 atom columns of 64 keys x 128 B apart)
            const uint64_t dv0 = sdesc(sbase + L::V, BN * 128, 1024);
            for (uint32_t jj = 0; jj < nblk && ok; jj++) {
                const uint32_t vb = jj % KVB, b = jj & 1;   // V buffer, P buffer
                if (!wait_cl(&v_full[vb], (jj / KVB) & 1)) break;
                const uint64_t dv = dv0 + vb * (uint32_t) (L::V_BUF / 16);
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    if (!wait_cl(&p_full[2 * t + b], (jj >> 1) & 1)) break;
                    tc_fence_after();
                    const uint32_t d = tmem + t * TS + 128;
                    const uint32_t pa = tmem + t * TS + BN + b * (BN / 2);
#pragma unroll
                    for (int ks = 0; ks < BN / 16; ks++)
                        tc2_mma_ts(d, pa + ks * 8, dv + (uint32_t) (ks * 2048 / 16), IDESC_PV, (jj > 0 || ks > 0) ? 1u : 0u);
                    tc2_commit(&pv_free[2 * t + b]);
                    if (jj + 1 == nblk) tc2_commit(&o_ready[t]);
                }
                if (!ok) break;
                tc2_commit(&v_free[vb]);
            }
        } else if (cr == 1 && lane == 0 && warp == 1) {
            // CTA 1: its Q tiles are in place
            if (wait(q_full, 0)) mbar_arrive_cl(lead(q_pair));
        }
        if (lane == 0) {
            // TMEM must not be released under MMAs still running: CTA 0's 1 + NT issuers commit to mma_done in both
            // CTAs (count 1 + NT), and the issuing warps' counterparts of both CTAs wait for it (bounded)
            if (cr == 0) tc2_commit(mma_done);
            const uint64_t drain = tmo > dec::DRAIN_NS ? tmo : dec::DRAIN_NS;
            if (!mbar_wait_bounded(mma_done, 0, drain, nullptr)) atomicCAS(p.status, ST_OK, ST_TIMEOUT_DRAIN);
        }
      }   // warp 3 with NT == 1: idle
    } else if (warp < (uint32_t) DQ0) {
        // ------------------------------------------------ softmax of pair tile t, this CTA's 128 rows
        if (NT == 2) asm volatile("setmaxnreg.inc.sync.aligned.u32 152;");
        if (D == 256) asm volatile("setmaxnreg.inc.sync.aligned.u32 168;");
        if (p.stall) wait(never, 0);   // runs out: records the timeout; the roles of both CTAs unwind (bounded waits)
        const int t = (int) (warp - SM0) / 4;
        const uint32_t wq = warp % 4;
        const uint32_t r = wq * 32 + lane;
        const uint32_t tl = tmem + ((wq * 32) << 16) + t * TS;
        // a warp whose 32 rows are all past the call's rows only keeps the barrier protocol (as in pa_prefill.cuh)
        const bool pad = NT == 1 && row0 + t * 2 * BM + cr * BM + wq * 32 >= p.rows;   // (NT = 1: registers, as there)
        float m_used = -INFINITY, l = 0.f;
        float m_row = -INFINITY;   // the row's exact maximum (log2 units); O and l are reported against it
        for (uint32_t j = 0; j < nblk; j++) {
            const uint32_t b = j & 1;
            if (!wait(&s_full[t], j & 1)) break;
            if (pad) {
                __syncwarp();
                if (lane == 0) { mbar_arrive_cl(lead(&s_empty[t])); mbar_arrive_cl(lead(&p_full[2 * t + b])); }
                continue;
            }
            tc_fence_after();
            float s[64];
            {
                float a[32], c[32];
                tmem_ld32(tl, a);
                tmem_ld32(tl + 32, c);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i++) { s[i] = a[i]; s[32 + i] = c[i]; }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cl(lead(&s_empty[t]));
            const int nvalid = (int) (job.nk - j * BN);
            if (nvalid < BN) {
#pragma unroll
                for (int i = 0; i < BN; i++)
                    if (i >= nvalid) s[i] = -INFINITY;
            }
            float mx = s[0];
#pragma unroll
            for (int i = 1; i + 1 < BN; i += 2) mx = max3(mx, s[i], s[i + 1]);
            mx = fmaxf(mx, s[BN - 1]);
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
            const uint64_t l2e2 = pack_f2(LOG2E, LOG2E), nm2 = pack_f2(-m_used, -m_used);
            uint64_t acc = pack_f2(0.f, 0.f);
            uint32_t ph[32];
#pragma unroll
            for (int i = 0; i < 32; i++) {
                float t0, t1;
                unpack_f2(fma_f2(pack_f2(s[2 * i], s[2 * i + 1]), l2e2, nm2), t0, t1);
                // every 4th pair on the FMA pipe, the rest on MUFU (measured: +3-5% over MUFU alone; every 2nd: -2%)
                float p0, p1;
                if (i % 4 == 3) ex2_pair_fma(t0, t1, p0, p1);
                else { p0 = ex2(t0); p1 = ex2(t1); }
                const uint64_t pp = pack_f2(p0, p1);
                acc = add_f2(acc, pp);
                ph[i] = pack_h2(p0, p1);
            }
            float sa, sb;
            unpack_f2(acc, sa, sb);
            const float sum = sa + sb;
            l = fmaf(l, alpha, sum);
            // as in pa_prefill.cuh: O is rescaled once P.V of block j-1 completed; P buffer b is free once P.V of
            // block j-2 completed (each wait names exactly one completion of its barrier)
            if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
                if (!wait(&pv_free[2 * t + (b ^ 1)], ((j - 1) >> 1) & 1)) break;
                tc_fence_after();
#pragma unroll
                for (int q = 0; q < D / 32; q++) {
                    float o[32];
                    tmem_ld32(tl + 128 + q * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] *= alpha;
                    tmem_st32(tl + 128 + q * 32, o);
                }
                tmem_wait_st();
            }
            if (j >= 2 && !wait(&pv_free[2 * t + b], ((j - 2) >> 1) & 1)) break;
            tmem_st32u(tl + BN + b * (BN / 2), ph);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cl(lead(&p_full[2 * t + b]));
        }
        // O and l moved from the lazy reference max m_used to the row's exact maximum (as in pa_prefill.cuh)
        if (ok && !pad && nblk > 0 && wait(&o_ready[t], 0)) {
            tc_fence_after();
            const uint32_t row = row0 + t * 2 * BM + cr * BM + r;
            const uint64_t orow = ((uint64_t) job.slot * p.nkv + h) * p.rows + row;
            const float fix = m_row > -INFINITY ? ex2(m_used - m_row) : 1.f;
#pragma unroll
            for (int q = 0; q < D / 32; q++) {
                float o[32];
                tmem_ld32(tl + 128 + q * 32, o);
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
        // ------------------------------------------------ dequantisers: (key, quant block) items (dq_item), one per lane
        // and pass (D = 128: one pass of each operand; D = 256: two)
        if (NT == 2) asm volatile("setmaxnreg.dec.sync.aligned.u32 80;");
        if (D == 256) asm volatile("setmaxnreg.dec.sync.aligned.u32 88;");
        const uint32_t dw = warp - DQ0;
        for (uint32_t j = 0; j < nblk; j++) {
            const uint32_t st = j % NS, b = j % KVB;
            if (!wait(&raw_full[st], (j / NS) & 1)) break;
            const uint32_t raw = sbase + L::RAW + st * L::RAW_STAGE;
#pragma unroll
            for (int kv = 0; kv < 2; kv++) {
                if (j >= KVB && !wait(kv == 0 ? &k_free[b] : &v_free[b], ((j / KVB) - 1) & 1)) break;
#pragma unroll
              for (int ps = 0; ps < NPASS; ps++) {
                uint32_t ql, qb, key;
                dq_item<D, NDQ>(kv, ps, dw, lane, cr, ql, qb, key);
                const uint32_t rb = raw + (kv == 0 ? 0u : (uint32_t) L::RAW_V) + key * RAWB;
                const uint32_t bo = hoff + GB * qb;
                const uint32_t w16 = bo & ~15u;
                const uint32_t ds = bo + 2;
                const uint32_t w0 = (ds - w16) / 4, shift = 8 * (ds % 4);
                const uint32_t dst = kv == 0 ? sbase + L::K + b * L::K_BUF + (ql / 2) * KH * 128
                                             : sbase + L::V + b * L::V_BUF + (ql / 2) * BN * 128;
                // the same offsets as dq_row / dq_chunk, written out (helper calls here cost the dequant role a spill
                // under its 80-register budget)
                const uint32_t kbase = dst + (key / 8) * 1024 + (key % 8) * 128;
                const uint32_t c0 = 4 * (ql % 2);
                const uint32_t s2 = lds16(rb + bo);
                const uint32_t sc2 = s2 | (s2 << 16);
                uint32_t W[12];
#pragma unroll
                for (int i = 0; i < (QUANT == 1 ? 3 : 2); i++)
                    lds128(rb + w16 + 16 * i, W[4 * i], W[4 * i + 1], W[4 * i + 2], W[4 * i + 3]);
                if (QUANT != 1) W[8] = W[9] = W[10] = W[11] = 0u;
                if (QUANT == 1) {
                    uint32_t A[8];
                    switch (w0) {
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
                        sts128(kbase + (((c0 + cc) ^ (key % 8)) * 16), h0, h1, h2, h3);
                    }
                } else {
                    uint32_t Dw[4];
                    switch (w0) {
#define PA_ALIGN4(W0)                                                                        \
    case W0:                                                                                 \
        _Pragma("unroll") for (int i = 0; i < 4; i++) Dw[i] = __funnelshift_r(W[W0 + i], W[W0 + i + 1], shift); \
        break;
                        PA_ALIGN4(0) PA_ALIGN4(1) PA_ALIGN4(2) PA_ALIGN4(3) default: PA_ALIGN4(4)
#undef PA_ALIGN4
                    }
                    uint32_t lo[8], hi[8];
                    const uint32_t m = 0x000F000Fu, magic = 0x64006400u, off8 = 0x64086408u;
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const uint32_t y = prmt(Dw[i], Dw[i], 0x3120u);
                        lo[2 * i] = hmul2(hsub2(and_or(y, m, magic), off8), sc2);
                        lo[2 * i + 1] = hmul2(hsub2(and_or(y >> 8, m, magic), off8), sc2);
                        hi[2 * i] = hmul2(hsub2(and_or(y >> 4, m, magic), off8), sc2);
                        hi[2 * i + 1] = hmul2(hsub2(and_or(y >> 12, m, magic), off8), sc2);
                    }
                    sts128(kbase + (((c0 + 0) ^ (key % 8)) * 16), lo[0], lo[1], lo[2], lo[3]);
                    sts128(kbase + (((c0 + 1) ^ (key % 8)) * 16), lo[4], lo[5], lo[6], lo[7]);
                    sts128(kbase + (((c0 + 2) ^ (key % 8)) * 16), hi[0], hi[1], hi[2], hi[3]);
                    sts128(kbase + (((c0 + 3) ^ (key % 8)) * 16), hi[4], hi[5], hi[6], hi[7]);
                }
              }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive_cl(lead(kv == 0 ? &k_full[b] : &v_full[b]));
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[st]);
        }
    }

    // every role of both CTAs ends here: no CTA exits while its peer can still arrive on its barriers or while MMAs
    // read its operands (warps 1 and 2 waited for mma_done), and both release TMEM together
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS) : "memory");
    }
}

}  // namespace pre
}  // namespace pa
