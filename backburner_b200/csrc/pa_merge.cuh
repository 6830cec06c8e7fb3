// pa_merge.cuh - log-sum-exp merge of unnormalised partials (O, m, l), and the final normalisation.
//
// Reference semantics:
//   pa_merge / pa_merge_big (phone-attn/pa-metal.mm:137-159, 490-524): M = max of the parts' m, parts with no keys
//     skipped, L = sum_c exp(m_c - M) l_c, O = sum_c exp(m_c - M) O_c; the fold bit also takes the result already in
//     (O, M, L) as one more part.
//   merge_partial (phone-attn/phone-attn.h:231-239): a part with l <= 0 contributes nothing.
//   attn_core's normalisation (phone-attn/phone-attn.h:651-655): O/l rounded to f16, lse = m + log l (-inf if l == 0).
// merge_kernel: one warp per output row (or 8 for calls with few rows and many parts); each lane owns hd/32
// consecutive head dims (float4 loads).
#pragma once
#include "pa_common.cuh"

namespace pa {
namespace mrg {

struct Params {
    const float *Op, *Mp, *Lp;   // parts: row R of part c of set s at Op + c * op_stride + (s * set_rows + R) * HD,
                                 // Mp / Lp + c * ml_stride + s * set_rows + R
    const uint32_t *c_range;     // [n_sets + 1]: parts [c_range[s], c_range[s+1]) of set s; null: [0, n_parts)
    uint32_t n_parts;
    uint64_t op_stride, ml_stride, set_rows;
    float *O, *M, *L;            // out: row R of set s at s * rows_per_set + R
    uint64_t rows_per_set;       // nkv * rows
    uint32_t n_sets;
    int fold;                    // 1: (O, M, L) already hold a partial to fold in
};

// SPLIT warps per output row (1: 8 rows per 256-thread block; 8: one row per block, for calls with few rows and many
// parts, where one warp walking every part of its row would leave the GPU idle). The row's parts are dealt out to its
// warps; each warp takes the maxima of its parts with its lanes in parallel, the row maximum M is agreed through shared
// memory, and every warp accumulates sum_c w_c O_c, sum_c w_c l_c against that same M, so the warps' sums simply add.
// Weights are computed 32 parts at a time (one per lane) and broadcast; the O loads of a batch do not depend on one
// another, and a part with l <= 0 (no keys) gets weight 0 and its O is not used.
template <int HD, int SPLIT>
__global__ void __launch_bounds__(256) merge_kernel(const Params p) {
    constexpr int V = HD / 32;          // floats per lane
    constexpr int RPB = 8 / SPLIT;      // rows per block
    __shared__ float s_m[8];
    __shared__ float s_l[8];
    __shared__ __align__(16) float s_acc[SPLIT > 1 ? 8 * HD : 4];
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32, sw = warp % SPLIT;
    const uint64_t gw = (uint64_t) blockIdx.x * RPB + warp / SPLIT;
    const bool active = gw < (uint64_t) p.n_sets * p.rows_per_set;
    const uint32_t s = active ? (uint32_t) (gw / p.rows_per_set) : 0;
    const uint64_t R = active ? gw % p.rows_per_set : 0;
    const uint32_t c0 = !active ? 0 : p.c_range ? p.c_range[s] : 0;
    const uint32_t c1 = !active ? 0 : p.c_range ? p.c_range[s + 1] : p.n_parts;
    const uint64_t orow = (uint64_t) s * p.rows_per_set + R;
    const uint64_t rr = (uint64_t) s * p.set_rows + R;

    // ---- the row maximum over the parts with keys (and the partial already in O, M, L when folding)
    float m_in = -INFINITY, l_in = 0.f;
    const bool fold = active && p.fold && sw == 0;
    if (fold) {
        m_in = p.M[orow];
        l_in = p.L[orow];
    }
    float M = (fold && l_in > 0.f) ? m_in : -INFINITY;
    for (uint32_t c = c0 + sw + SPLIT * lane; c < c1; c += 32 * SPLIT) {
        const uint64_t pr = (uint64_t) c * p.ml_stride + rr;
        if (p.Lp[pr] > 0.f) M = fmaxf(M, p.Mp[pr]);
    }
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
    if (SPLIT > 1) {
        if (lane == 0) s_m[warp] = M;
        __syncthreads();
        const uint32_t w0 = (warp / SPLIT) * SPLIT;
#pragma unroll
        for (int w = 0; w < SPLIT; w++) M = fmaxf(M, s_m[w0 + w]);
    }

    // ---- sum_c w_c O_c and sum_c w_c l_c against M
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; i++) acc[i] = 0.f;
    float Ls = 0.f;   // this lane's share of the weighted l
    if (fold && l_in > 0.f) {
        const float w = ex2((m_in - M) * LOG2E);
        if (lane == 0) Ls = w * l_in;
        const float4 *src = reinterpret_cast<const float4 *>(p.O + orow * HD + lane * V);
#pragma unroll
        for (int i = 0; i < V / 4; i++) {
            const float4 x = src[i];
            acc[4 * i] = w * x.x; acc[4 * i + 1] = w * x.y; acc[4 * i + 2] = w * x.z; acc[4 * i + 3] = w * x.w;
        }
    }
    for (uint32_t cb = c0 + sw; cb < c1; cb += 32 * SPLIT) {
        const uint32_t c = cb + SPLIT * lane;
        float w = 0.f;
        if (c < c1) {
            const uint64_t pr = (uint64_t) c * p.ml_stride + rr;
            const float lc = p.Lp[pr];
            if (lc > 0.f) {
                w = ex2((p.Mp[pr] - M) * LOG2E);
                Ls = fmaf(w, lc, Ls);
            }
        }
        const uint32_t nb = min(32u, (c1 - cb + SPLIT - 1) / SPLIT);
#pragma unroll 4
        for (uint32_t j = 0; j < nb; j++) {
            const float wj = __shfl_sync(0xffffffffu, w, j);
            const float4 *src =
                reinterpret_cast<const float4 *>(p.Op + (uint64_t) (cb + SPLIT * j) * p.op_stride + rr * HD + lane * V);
#pragma unroll
            for (int i = 0; i < V / 4; i++) {
                const float4 x = src[i];
                if (wj != 0.f) {   // a part without keys (l <= 0) may hold anything in O
                    acc[4 * i] = fmaf(wj, x.x, acc[4 * i]);
                    acc[4 * i + 1] = fmaf(wj, x.y, acc[4 * i + 1]);
                    acc[4 * i + 2] = fmaf(wj, x.z, acc[4 * i + 2]);
                    acc[4 * i + 3] = fmaf(wj, x.w, acc[4 * i + 3]);
                }
            }
        }
    }
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, x);
    if (SPLIT > 1) {
        // the row's warps add their sums through shared memory; the row's first warp writes the result
        float4 *mine = reinterpret_cast<float4 *>(s_acc + warp * HD + lane * V);
#pragma unroll
        for (int i = 0; i < V / 4; i++) mine[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
        if (lane == 0) s_l[warp] = Ls;
        __syncthreads();
        if (sw != 0) return;
        for (int w = 1; w < SPLIT; w++) {
            const float4 *o = reinterpret_cast<const float4 *>(s_acc + (warp + w) * HD + lane * V);
#pragma unroll
            for (int i = 0; i < V / 4; i++) {
                const float4 x = o[i];
                acc[4 * i] += x.x; acc[4 * i + 1] += x.y; acc[4 * i + 2] += x.z; acc[4 * i + 3] += x.w;
            }
            Ls += s_l[warp + w];
        }
    }
    if (!active) return;
    float4 *dst = reinterpret_cast<float4 *>(p.O + orow * HD + lane * V);
#pragma unroll
    for (int i = 0; i < V / 4; i++) dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
    if (lane == 0) {
        p.M[orow] = Ls > 0.f ? M : -INFINITY;
        p.L[orow] = Ls;
    }
}

// One warp's merge of parts [c0, c1) of one row: part c's row at Op + c * op_stride + rr * HD, its m and l at
// Mp / Lp + c * ml_stride + rr. Returns sum_c w_c O_c (this lane's HD/32 dims), M and sum_c w_c l_c, w_c =
// exp(m_c - M), parts with l <= 0 skipped (M = -inf, L = 0 when none has keys). As merge_kernel's one-warp path.
template <int HD>
__device__ __forceinline__ void merge_row(const float *Op, const float *Mp, const float *Lp, uint64_t op_stride,
                                          uint64_t ml_stride, uint64_t rr, uint32_t c0, uint32_t c1, uint32_t lane,
                                          float (&acc)[HD / 32], float &M, float &L) {
    constexpr int V = HD / 32;
    M = -INFINITY;
    for (uint32_t c = c0 + lane; c < c1; c += 32) {
        const uint64_t pr = (uint64_t) c * ml_stride + rr;
        if (Lp[pr] > 0.f) M = fmaxf(M, Mp[pr]);
    }
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
#pragma unroll
    for (int i = 0; i < V; i++) acc[i] = 0.f;
    float Ls = 0.f;
    for (uint32_t cb = c0; cb < c1; cb += 32) {
        const uint32_t c = cb + lane;
        float w = 0.f;
        if (c < c1) {
            const uint64_t pr = (uint64_t) c * ml_stride + rr;
            const float lc = Lp[pr];
            if (lc > 0.f) {
                w = ex2((Mp[pr] - M) * LOG2E);
                Ls = fmaf(w, lc, Ls);
            }
        }
        const uint32_t nb = min(32u, c1 - cb);
#pragma unroll 4
        for (uint32_t j = 0; j < nb; j++) {
            const float wj = __shfl_sync(0xffffffffu, w, j);
            const float4 *src = reinterpret_cast<const float4 *>(Op + (uint64_t) (cb + j) * op_stride + rr * HD + lane * V);
#pragma unroll
            for (int i = 0; i < V / 4; i++) {
                const float4 x = src[i];
                if (wj != 0.f) {
                    acc[4 * i] = fmaf(wj, x.x, acc[4 * i]);
                    acc[4 * i + 1] = fmaf(wj, x.y, acc[4 * i + 1]);
                    acc[4 * i + 2] = fmaf(wj, x.z, acc[4 * i + 2]);
                    acc[4 * i + 3] = fmaf(wj, x.w, acc[4 * i + 3]);
                }
            }
        }
    }
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, x);
    L = Ls;
}

// ---------------------------------------------------------------- the peer-store exchange of position shards
// One kernel per call on every rank (one process per GPU): block b merges rows [8b, 8b+8) of this rank's chunk partials
// (the plan's slots), stores them into every rank's receive area over NVLink (packed as one rank's part: O [rows][HD],
// m [rows], l [rows]), publishes `epoch` in each rank's flag for (this rank, block b) with a system-scope release, waits
// (bounded) until every rank has published block b of this call in this rank's flags, and folds the ranks' rows into
// O, M, L. Blocks store before they wait, so a block waits only for blocks that store first on the other GPUs.
struct XParams {
    const float *Op, *Mp, *Lp;          // this rank's chunk partials (plan slots), as merge_kernel's Params
    const uint32_t *c_range;            // [n_sets + 1]
    uint64_t op_stride, ml_stride, rows_per_set;
    uint32_t n_sets;
    float *const *push;                 // [world]: rank r's receive area, this rank's part (half 0)
    uint64_t push_off;                  // floats from half 0 to this call's half
    unsigned long long *const *push_flag;   // [world]: rank r's flags of source = this rank, [blocks]
    const float *recv;                  // this rank's receive area, this call's half: rank r's part at recv + r * cap
    const unsigned long long *flags;    // this rank's flags [world][blocks_cap]
    uint64_t cap, blocks_cap;
    unsigned long long epoch;           // this call's number (1, 2, ...)
    uint32_t world;
    float *O, *M, *L;
    int *status;
    uint64_t timeout_ns;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

template <int HD>
__global__ void __launch_bounds__(256) shard_exchange_kernel(const XParams p) {
    constexpr int V = HD / 32;
    const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint64_t rows = (uint64_t) p.n_sets * p.rows_per_set;
    const uint64_t row = (uint64_t) blockIdx.x * 8 + warp;
    const bool active = row < rows;
    float acc[V], M = -INFINITY, L = 0.f;
    if (active) {
        const uint32_t s = (uint32_t) (row / p.rows_per_set);
        merge_row<HD>(p.Op, p.Mp, p.Lp, p.op_stride, p.ml_stride, row % p.rows_per_set, p.c_range[s], p.c_range[s + 1],
                      lane, acc, M, L);
        for (uint32_t r = 0; r < p.world; r++) {
            float *base = p.push[r] + p.push_off;
            float4 *dst = reinterpret_cast<float4 *>(base + row * HD + lane * V);
#pragma unroll
            for (int i = 0; i < V / 4; i++) dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
            if (lane == 0) {
                base[rows * HD + row] = L > 0.f ? M : -INFINITY;
                base[rows * HD + rows + row] = L;
            }
        }
    }
    __syncthreads();   // the block's stores, then (cumulative system-scope fence) its flag in every rank
    if (threadIdx.x < p.world) {
        __threadfence_system();
        st_release_sys(p.push_flag[threadIdx.x] + blockIdx.x, p.epoch);
    }
    __shared__ int s_go;
    if (threadIdx.x == 0) {
        bool go = *(volatile int *) p.status == ST_OK;   // a call that already failed waits no further
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t r = 0; go && r < p.world; r++) {
            const unsigned long long *f = p.flags + (uint64_t) r * p.blocks_cap + blockIdx.x;
            for (uint32_t it = 0; ld_acquire_sys(f) < p.epoch; it++) {
                if ((it & 63) == 63 && globaltimer_ns() - t0 > p.timeout_ns) {
                    atomicCAS(p.status, ST_OK, ST_TIMEOUT_PEER);
                    go = false;
                    break;
                }
            }
        }
        s_go = go;
    }
    __syncthreads();
    if (!s_go || !active) return;
    merge_row<HD>(p.recv, p.recv + rows * HD, p.recv + rows * HD + rows, p.cap, p.cap, row, 0, p.world, lane, acc, M, L);
    float4 *dst = reinterpret_cast<float4 *>(p.O + row * HD + lane * V);
#pragma unroll
    for (int i = 0; i < V / 4; i++) dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
    if (lane == 0) {
        p.M[row] = L > 0.f ? M : -INFINITY;
        p.L[row] = L;
    }
}

// O/l -> f16, lse = m + log(l); rows with l == 0 give O = 0, lse = -inf
template <int HD>
__global__ void __launch_bounds__(256) normalize_kernel(const float *O, const float *M, const float *L, uint64_t n_rows,
                                                        uint16_t *Oh, float *lse) {
    constexpr int V = HD / 32;
    const uint64_t r = (uint64_t) blockIdx.x * 8 + threadIdx.x / 32;
    const uint32_t lane = threadIdx.x % 32;
    if (r >= n_rows) return;
    const float l = L[r];
    const float inv = l > 0.f ? 1.0f / l : 0.0f;
#pragma unroll
    for (int i = 0; i < V; i += 2) {
        const uint32_t h2 = pack_h2(O[r * HD + lane * V + i] * inv, O[r * HD + lane * V + i + 1] * inv);
        *reinterpret_cast<uint32_t *>(Oh + r * HD + lane * V + i) = h2;
    }
    if (lane == 0) lse[r] = l > 0.f ? M[r] + logf(l) : -INFINITY;
}

// The host's co-attention fold of a normalised reply (phone-attn/phone-attn.h:18-20: "O_unnorm = O, S = 1, M = lse"):
// the reply row (f16 O = O/l, lse = m + log l) is the part (O, m = lse, l = 1), merged into the unnormalised partial
// already in (O, M, L) by merge_partial's rule (phone-attn/phone-attn.h:231-239): a reply with lse = -inf (no keys)
// adds nothing; a partial with L <= 0 is replaced. One warp per row.
template <int HD>
__global__ void __launch_bounds__(256) fold_reply_kernel(const uint16_t *Oh, const float *lse, uint64_t n_rows, float *O,
                                                         float *M, float *L) {
    constexpr int V = HD / 32;
    const uint64_t r = (uint64_t) blockIdx.x * 8 + threadIdx.x / 32;
    const uint32_t lane = threadIdx.x % 32;
    if (r >= n_rows) return;
    const float mr = lse[r];
    if (!(mr > -INFINITY)) return;
    const float m_in = M[r], l_in = L[r];
    const bool keep = l_in > 0.f;
    const float Mx = keep ? fmaxf(m_in, mr) : mr;
    const float a = keep ? ex2((m_in - Mx) * LOG2E) : 0.f, b = ex2((mr - Mx) * LOG2E);
    float *o = O + r * HD + lane * V;
    const uint16_t *h = Oh + r * HD + lane * V;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const float x = __half2float(__ushort_as_half(h[i]));
        o[i] = keep ? fmaf(o[i], a, x * b) : x * b;
    }
    __syncwarp();
    if (lane == 0) {
        M[r] = Mx;
        L[r] = keep ? fmaf(l_in, a, b) : b;
    }
}

// The all-reduce exchange of position shards: once M holds each row's maximum over all ranks' partials, this rank's
// partial (O, m, l) is moved to it, w = exp(m - M), so that the ranks' partials add up to the merge of pa_merge /
// merge_partial: O = sum_r w_r O_r, l = sum_r w_r l_r (a rank without keys in the row has l = 0 and adds nothing; a row
// no rank has keys for keeps O = 0, l = 0, M = -inf). In place; one warp per row.
template <int HD>
__global__ void __launch_bounds__(256) rescale_to_kernel(float *O, const float *m, float *l, const float *M,
                                                         uint64_t n_rows) {
    constexpr int V = HD / 32;
    const uint64_t r = (uint64_t) blockIdx.x * 8 + threadIdx.x / 32;
    const uint32_t lane = threadIdx.x % 32;
    if (r >= n_rows) return;
    const float lr = l[r], mr = m[r], Mr = M[r];
    const float w = (lr > 0.f && Mr > -INFINITY) ? ex2((mr - Mr) * LOG2E) : 0.f;
    float4 *o = reinterpret_cast<float4 *>(O + r * HD + lane * V);
#pragma unroll
    for (int i = 0; i < V / 4; i++) {
        const float4 x = o[i];
        o[i] = make_float4(w * x.x, w * x.y, w * x.z, w * x.w);
    }
    __syncwarp();
    if (lane == 0) l[r] = w * lr;
}

// f16(q * scale) for n fp32 values (scripts/sme/sme_attn.c:276-280; phone-attn/phone-attn.h:595-599)
__global__ void scale_q_kernel(const float *Q, float scale, uint64_t n, uint16_t *Qs) {
    for (uint64_t i = (uint64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t) gridDim.x * blockDim.x)
        Qs[i] = __half_as_ushort(__float2half_rn(Q[i] * scale));
}

}  // namespace mrg
}  // namespace pa
