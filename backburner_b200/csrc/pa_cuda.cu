// pa_cuda.cu - libpacuda.so: the C ABI of include/pa_cuda.h over the sm_100a kernels (pa_decode.cuh, pa_merge.cuh).
// Host side: contexts, plans (the split of a call into chunk jobs), the pa::engine page/begin/end path, and the
// device status word that bounded in-kernel waits report into.
#include "pa_cuda.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <mutex>
#include <thread>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "pa_decode.cuh"
#include "pa_merge.cuh"
#include "pa_prefill.cuh"
#include "pa_prefill_pair.cuh"

namespace {

constexpr int kMaxSmem = 227 * 1024;
// query rows per KV head from which the tcgen05 kernels are used: they dequantise each key block once for all rows,
// where the split-K kernel repeats it per 8-row group. Measured crossover (8 KV heads x 4 layers x 32,768 Q8_0 keys,
// GB/s split-K vs the single-CTA tcgen05 kernel): hd 128: 8 rows 3,636 vs 2,569, 12 rows 2,095 vs 2,558, 16 rows 2,066
// vs 2,558 (4 KV heads: 8 rows 2,882 vs 2,329, 12 rows 1,910 vs 2,328); hd 256: 8 rows 4,267 vs 3,547, 12 rows 2,259 vs
// 3,535, 16 rows 2,177 vs 3,545 (4 KV heads: 8 rows 3,463 vs 3,247, 12 rows 2,230 vs 3,238). One 8-row group stays on
// the split-K kernel.
constexpr uint32_t kPrefillMinRows128 = 9, kPrefillMinRows256 = 9;
// ... and from which the hd-128 calls run on CTA pairs: past 256 rows the single-CTA kernel starts a second, partly
// filled tile. Measured (8 KV heads x 4 layers x 65,536 Q8_0 keys, TFLOP/s single vs pair): 256 rows 676 vs 558,
// 320 510 vs 549, 384 608 vs 643, 448 667 vs 694, 512 751 vs 784
constexpr uint32_t kPairMinRows = 257;
// ... and up to which hd-256 calls run on the single-CTA kernel with one 128-row tile; above, on CTA pairs. Measured
// (8 KV heads x 4 layers x 32,768 Q8_0 keys, us single vs pair): 48 rows 166 vs 305, 128 rows 174 vs 305, 144 rows 327
// vs 311, 256 rows 335 vs 317
constexpr uint32_t kSingle256MaxRows = 128;
// Per-job overhead of the decode kernel in keys, for the job-size model of pa_cuda_plan_create. Fitted on B200 to
// config-1 runs of the current kernel (kernel ms, 64 layers): 131,072 keys per layer as 2,048-key jobs 3.618, 4,096
// 3.600, 8,192 3.708, 14,592 3.684; 16,384 keys per layer (an 8-way shard) as 1,024 0.491, 1,856 0.487, 2,048 0.535,
// 4,096 0.532. (A persistent variant, each CTA taking several jobs through one stage stream, measured no better.)
constexpr uint32_t kDecodeJobOverhead = 48;
// Per-job overhead of the tcgen05 kernels in keys (a CTA's set-up is ~5-10 us, ~64 keys of an hd-256 block a us), for the
// same model. Measured on the server's 8-token ATTN (hd 256, 4 KV heads, 48 rows, 32,768 keys): 1,024-key jobs 58.6 us
// (kernel), 2,048-key jobs 51.6 us.
constexpr uint32_t kPrefillJobOverhead = 512;

struct Plan;

// pa::engine calls: plans are kept per call shape (a layer's pages, its key counts, the geometry), so the per-layer
// calls of a decode step reuse their job lists and partial buffers instead of allocating them every call; a plan
// armed for the next call (pa_cuda_arm) also holds a CUDA graph of the whole call.
constexpr size_t kEngCache = 256;                 // plans at most
constexpr size_t kEngCacheBytes = 1ull << 30;     // and at most this much plan scratch (partials, job lists)
struct EngEntry {
    std::vector<uint64_t> key;           // geometry, groups, packed tokens, kernel choice, QK arithmetic, then (k, v,
                                         // nkeys) per page
    pa_cuda_plan *plan = nullptr;
    cudaGraphExec_t graph = nullptr;     // Q upload, kernels, result readback (captured by pa_cuda_arm)
    uint64_t graph_launches = 0;         // kernel launches one replay makes
    uint64_t used = 0;                   // LRU tick
};

}  // namespace

struct pa_cuda_ctx {
    int device = 0;
    int n_sm = 148;
    cudaStream_t stream = nullptr;
    int *d_status = nullptr;
    int *h_status = nullptr;      // pinned: the status word read back by pa_cuda_status
    uint64_t timeout_ns = 2000000000ull;
    uint64_t launches = 0;
    int stall_test = 0;
    int kernel_choice = 0;   // 0 auto, 1 split-K mma.sync kernel, 2 tcgen05 kernel (one CTA), 3 tcgen05 on CTA pairs
    int qk_domain = PA_CUDA_QK_F16;   // PA_CUDA_QK_INT8: int8-domain QK (Q8_0 rows, split-K kernel)
    std::string err;
    // pa::engine state (begin/end)
    pa_cuda_plan *eng_plan = nullptr;      // the current call's plan (owned by eng_cache)
    std::vector<EngEntry> eng_cache;
    uint64_t eng_tick = 0, eng_graph_calls = 0;
    std::vector<pa_cuda_seg> eng_segs;
    // keys of each page (by its K pointer) already prefetched to the device: a call prefetches only what the host wrote
    // since (pages new to the engine, rows appended; a page that shrank is prefetched whole)
    std::unordered_map<uintptr_t, uint32_t> eng_resident;
    uint16_t *h_q = nullptr;      // pinned staging
    float *h_out = nullptr;       // pinned staging: O, then m, then l, then the call's status word
    size_t h_q_bytes = 0, h_out_bytes = 0;
    uint16_t *d_q = nullptr;
    float *d_out = nullptr;
    size_t d_q_bytes = 0, d_out_bytes = 0;
    cudaEvent_t ev_begin = nullptr, ev_end = nullptr;
    std::chrono::steady_clock::time_point t_begin;
    int eng_ng = 0, eng_nt = 0, eng_rows = 0, eng_nkv = 0, eng_hd = 0;
    bool eng_active = false;
    double last_exec_ms = 0;
    // position shards over NCCL: this rank's packed (O, m, l) and every rank's
    float *d_shard = nullptr, *d_gathered = nullptr;
    size_t d_shard_bytes = 0, d_gathered_bytes = 0;
    int shard_exchange = 0;          // 0 by size, 1 all-gather + fold, 2 max / sum all-reduces
    int shard_groups = 0;            // 0 by size; else output-set groups whose exchange overlaps the next group's kernels
    int shard_last_mode = 0, shard_last_groups = 0;   // what the last shard call used
    uint32_t shard_timeout_ms = 0;   // > 0: the shard call waits for its exchange, bounded (abort on overrun)
    cudaStream_t xstream = nullptr;  // exchange stream of the pipelined shard call
    std::vector<cudaEvent_t> xev;    // [group] the group's partial is packed; back: the exchange finished
};

struct pa_cuda_plan {
    pa_cuda_ctx *ctx = nullptr;
    pa_cuda_shape sh{};
    uint32_t n_sets = 0, n_jobs = 0, n_slots = 0;
    pa::dec::Job *d_jobs = nullptr;
    uint32_t *d_crange = nullptr;
    std::vector<uint32_t> crange;       // host copy: jobs (= slots) [crange[s], crange[s+1]) belong to set s
    float *d_op = nullptr, *d_mp = nullptr, *d_lp = nullptr;
    size_t scratch = 0;
    // decode launch shape
    uint32_t hg = 1, rgc = 1, n_rg = 1, n_consumers = 1, row = 0, gs = 0, grid_y = 1, w = 8;
    size_t smem = 0;
    // tcgen05 path (many query rows per KV head, hd 128): tiles of NT x 128 rows (NT x 256 on a CTA pair), tensor
    // maps of the K/V segments
    bool prefill = false, pair = false;
    bool qk_i8 = false;   // split-K kernel with the int8-domain QK (decode_kernel<HD, 3, W>)
    int nt = 1;
    uint32_t n_rt = 0;
    CUtensorMap *d_maps = nullptr;
    // profiling: event pairs around the decode kernel of each run (a ring, summed by pa_cuda_plan_kernel_ms)
    bool profile = false;
    std::vector<cudaEvent_t> ev;
    uint32_t ev_used = 0;
};

namespace {

int fail(pa_cuda_ctx *ctx, int code, const std::string &msg) {
    if (ctx) ctx->err = msg;
    return code;
}
int cuda_fail(pa_cuda_ctx *ctx, cudaError_t e, const char *what) {
    return fail(ctx, PA_CUDA_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
#define PA_CK(call, what)                                    \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return cuda_fail(ctx, e_, what); \
    } while (0)

cudaStream_t pick(pa_cuda_ctx *ctx, void *stream) { return stream ? (cudaStream_t) stream : ctx->stream; }

size_t head_bytes(uint32_t quant, uint32_t hd) {
    return quant == PA_CUDA_Q8_0 ? hd / 32 * 34 : quant == PA_CUDA_Q4_0 ? hd / 32 * 18 : hd * 2;
}

int check_shape(pa_cuda_ctx *ctx, const pa_cuda_shape *sh) {
    if (!sh) return fail(ctx, PA_CUDA_EINVAL, "shape is null");
    if (sh->hd != 128 && sh->hd != 256) return fail(ctx, PA_CUDA_EUNSUPPORTED, "hd must be 128 or 256");
    if (sh->quant != PA_CUDA_F16 && sh->quant != PA_CUDA_Q8_0 && sh->quant != PA_CUDA_Q4_0)
        return fail(ctx, PA_CUDA_EUNSUPPORTED, "quant must be F16 (0), Q8_0 (1) or Q4_0 (2)");
    if (sh->nkv < 1 || sh->nkv > 64) return fail(ctx, PA_CUDA_EINVAL, "nkv out of range");
    if (sh->rows < 1) return fail(ctx, PA_CUDA_EINVAL, "rows must be >= 1");
    if (sh->hb != head_bytes(sh->quant, sh->hd)) return fail(ctx, PA_CUDA_EINVAL, "hb does not match quant/hd");
    if (sh->rs < (uint64_t) sh->nkv * sh->hb) return fail(ctx, PA_CUDA_EINVAL, "rs < nkv * hb");
    if (sh->rs % 16) return fail(ctx, PA_CUDA_EUNSUPPORTED, "rs must be a multiple of 16 bytes");
    return PA_CUDA_OK;
}

// launch shape of the decode kernel for a geometry
int plan_decode_shape(pa_cuda_ctx *ctx, pa_cuda_plan *p) {
    const pa_cuda_shape &sh = p->sh;
    // warps per CTA (the kernel instance): 8, except 4 at hd 256 when 8 KV heads cannot share a CTA
    p->w = (sh.hd == 256 && sh.nkv % 8) ? 4 : 8;
    const uint32_t maxw = p->w;
    const int nst = pa::dec::nstage((int) sh.hd);
    p->n_rg = (sh.rows + 7) / 8;
    // shared memory of NSTAGE stages of key pairs for head-group rows of `row` bytes (pairs padded to an odd number of
    // 16-byte units)
    auto pair_stride = [](uint32_t row) { uint32_t gs = 2 * row; return (gs / 16) % 2 == 0 ? gs + 16 : gs; };
    auto smem_for = [&sh, nst](uint32_t gs) {
        return (size_t) nst * pa::dec::stage_keys((int) sh.hd) * gs + pa::dec::SMEM_SLACK + (nst + 3) * 8 + 2 * nst * 4 + 16;
    };
    // the largest head group that divides nkv, gives 16-byte aligned rows and fits shared memory
    uint32_t hg = 0;
    bool aligned = false;
    for (uint32_t c = std::min(sh.nkv, maxw); c >= 1; c--) {
        if (sh.nkv % c) continue;
        if ((c * sh.hb) % 16) continue;
        aligned = true;
        if (smem_for(pair_stride((uint32_t) (c * sh.hb))) > (size_t) kMaxSmem) continue;
        hg = c;
        break;
    }
    if (!hg && !aligned) return fail(ctx, PA_CUDA_EUNSUPPORTED, "no head grouping gives 16-byte aligned rows (nkv * hb)");
    if (!hg) return fail(ctx, PA_CUDA_EUNSUPPORTED, "rows of this head group do not fit shared memory");
    p->hg = hg;
    p->rgc = std::min(p->n_rg, maxw / hg);
    const uint32_t S = hg * p->rgc;
    p->n_consumers = S;   // one warp per (head, row group) stream
    p->grid_y = (sh.nkv / hg) * ((p->n_rg + p->rgc - 1) / p->rgc);
    p->row = (uint32_t) (hg * sh.hb);                  // a multiple of 16 by the choice of hg
    p->gs = pair_stride(p->row);
    p->smem = smem_for(p->gs);
    return PA_CUDA_OK;
}

// ------------------------------------------------------------------ tensor maps (driver entry point, no -lcuda)
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return (PFN_cuTensorMapEncodeTiled_v12000) f;
    }();
    return fn;
}
// quantised rows of one segment as a 2-D u8 tensor {rs bytes, nk keys}; a box is one head's 16-byte-aligned window
// (16-bit elements: a 272-byte hd-256 window is 136 elements, within TMA's 256-element box limit; rs % 16 == 0)
bool map_rows(CUtensorMap *m, const void *base, uint64_t rs, uint32_t nk, uint32_t raw_bytes, uint32_t box_keys) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {rs / 2, nk};
    const cuuint64_t strides[1] = {rs};
    const cuuint32_t box[2] = {raw_bytes / 2, box_keys};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// Qs [all rows][hd] f16 with the 128-byte swizzle of the UMMA operand layout; a box is 64 dims x 128 rows
bool map_q(CUtensorMap *m, const void *Qs, uint64_t n_rows, uint32_t hd) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {hd, n_rows};
    const cuuint64_t strides[1] = {(cuuint64_t) hd * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t) pa::pre::BM};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(Qs), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int Q, int NT, int D = 128>
cudaError_t launch_prefill(const pa_cuda_plan *p, uint32_t nj, const CUtensorMap &tq, const pa::pre::Params &prm,
                           cudaStream_t st) {
    auto kern = pa::pre::prefill_kernel<Q, NT, D>;
    constexpr int smem = pa::pre::Smem<Q, NT, D>::TOTAL + 1024;   // + alignment slack for the 1024-byte operand tiles
    static_assert(smem <= 227 * 1024, "shared memory of a CTA");
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(nj * p->sh.nkv * p->n_rt);   // CTA = (row-tile group, head, job), row-tile group fastest
    kern<<<grid, 32 * pa::pre::cta_warps(NT), smem, st>>>(tq, prm);
    return cudaGetLastError();
}
// the CTA-pair kernel: clusters of 2 CTAs along x, one cluster per job
template <int Q, int NT, int D>
cudaError_t launch_prefill_pair(const pa_cuda_plan *p, uint32_t nj, const CUtensorMap &tq, const pa::pre::Params &prm,
                                cudaStream_t st) {
    auto kern = pa::pre::prefill_pair_kernel<Q, NT, D>;
    constexpr int smem = pa::pre::PairSmem<Q, NT, D>::TOTAL + 1024;
    static_assert(smem <= 227 * 1024, "shared memory of a CTA");
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * nj * p->sh.nkv * p->n_rt);   // cluster = (row-tile group, head, job), row-tile group fastest
    cfg.blockDim = dim3(32 * (4 + 4 * NT + pa::pre::pair_dq_warps(D)));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, tq, prm);
    return e != cudaSuccess ? e : cudaGetLastError();
}

// grid x: CTAs along the jobs (each takes jobs x, x + grid_x, ...; at most prm.n_jobs)
template <int HD, int Q, int W>
cudaError_t launch_decode(const pa_cuda_plan *p, uint32_t grid_x, const pa::dec::Params &prm, cudaStream_t st) {
    auto kern = pa::dec::decode_kernel<HD, Q, W>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) p->smem);
    if (e != cudaSuccess) return e;
    dim3 grid(grid_x, p->grid_y);
    kern<<<grid, 32 * p->n_consumers, p->smem, st>>>(prm);
    return cudaGetLastError();
}
// CTAs of a plan's decode-kernel instance that fit one SM at once (registers, shared memory, threads)
template <int HD, int Q, int W>
int decode_regs() {
    cudaFuncAttributes a{};
    return cudaFuncGetAttributes(&a, pa::dec::decode_kernel<HD, Q, W>) == cudaSuccess ? a.numRegs : 128;
}
template <int HD, int W>
int decode_regs_q(uint32_t q, bool i8) {
    return q == PA_CUDA_Q8_0 ? (i8 ? decode_regs<HD, 3, W>() : decode_regs<HD, 1, W>())
         : q == PA_CUDA_Q4_0 ? decode_regs<HD, 2, W>() : decode_regs<HD, 0, W>();
}
int decode_ctas_per_sm(const pa_cuda_plan *p) {
    const uint32_t hd = p->sh.hd, q = p->sh.quant;
    const bool i8 = p->qk_i8;
    const int regs = hd == 128 ? decode_regs_q<128, 8>(q, i8)
                   : p->w == 4 ? decode_regs_q<256, 4>(q, i8) : decode_regs_q<256, 8>(q, i8);
    const int threads = 32 * (int) p->n_consumers;
    const int by_regs = 65536 / std::max(1, threads * ((regs + 7) / 8 * 8));
    const int by_smem = (int) ((228u * 1024u) / (p->smem + 1024));
    const int by_threads = 2048 / std::max(1, threads);
    return std::max(1, std::min(std::min(by_regs, by_smem), std::min(by_threads, 32)));
}
// the decode-kernel instance of a geometry (hd 128 / 256; f16, Q8_0 or Q4_0 rows, Q8_0 with the int8-domain QK; warps
// per CTA)
template <int HD, int W>
cudaError_t launch_decode_q(const pa_cuda_plan *p, uint32_t nj, const pa::dec::Params &prm, cudaStream_t st, uint32_t quant) {
    return quant == PA_CUDA_Q8_0 ? (p->qk_i8 ? launch_decode<HD, 3, W>(p, nj, prm, st) : launch_decode<HD, 1, W>(p, nj, prm, st))
         : quant == PA_CUDA_Q4_0 ? launch_decode<HD, 2, W>(p, nj, prm, st) : launch_decode<HD, 0, W>(p, nj, prm, st);
}
cudaError_t launch_decode_any(const pa_cuda_plan *p, uint32_t nj, const pa::dec::Params &prm, cudaStream_t st, uint32_t hd,
                              uint32_t quant) {
    if (hd == 128) return launch_decode_q<128, 8>(p, nj, prm, st, quant);
    return p->w == 4 ? launch_decode_q<256, 4>(p, nj, prm, st, quant) : launch_decode_q<256, 8>(p, nj, prm, st, quant);
}

// The merge over the parts of each output row: 8 warps per row when the rows are few (8 warps each would still fit the
// SMs twice over) and the sets have many parts, else one warp per row
template <int HD>
cudaError_t launch_merge(const pa::mrg::Params &mp, cudaStream_t st, int n_sm) {
    const uint64_t rows = (uint64_t) mp.n_sets * mp.rows_per_set;
    if (rows == 0) return cudaSuccess;
    const uint64_t parts_per_set = mp.n_sets ? ((uint64_t) mp.n_parts + mp.n_sets - 1) / mp.n_sets : 0;
    if (rows * 8 <= (uint64_t) n_sm * 128 && parts_per_set >= 8)
        pa::mrg::merge_kernel<HD, 8><<<(unsigned) rows, 256, 0, st>>>(mp);
    else
        pa::mrg::merge_kernel<HD, 1><<<(unsigned) ((rows + 7) / 8), 256, 0, st>>>(mp);
    return cudaGetLastError();
}

// The plan's output sets [s0, s1): the attention kernel over their jobs (jobs are grouped by set, so they are the
// contiguous range [crange[s0], crange[s1])) and the merge of their slots into O, m, l, which point at set s0's rows.
// Qs is the whole call's Q (the kernels address it by each job's absolute set).
int run_attention_sets(pa_cuda_plan *p, const uint16_t *Qs, cudaStream_t st, uint32_t s0, uint32_t s1) {
    pa_cuda_ctx *ctx = p->ctx;
    const pa_cuda_shape &sh = p->sh;
    const uint32_t j0 = p->crange[s0], nj = p->crange[s1] - j0;
    if (nj > 0 && p->prefill) {
        CUtensorMap tq;
        if (!map_q(&tq, Qs, (uint64_t) p->n_sets * sh.nkv * sh.rows, sh.hd))
            return fail(ctx, PA_CUDA_ECUDA, "cuTensorMapEncodeTiled (Q) failed");
        pa::pre::Params prm{};
        prm.jobs = p->d_jobs + j0;
        prm.Qs = Qs;
        prm.kv_maps = p->d_maps;
        prm.Op = p->d_op;
        prm.Mp = p->d_mp;
        prm.Lp = p->d_lp;
        prm.status = ctx->d_status;
        prm.rs = sh.rs;
        prm.hb = sh.hb;
        prm.nkv = sh.nkv;
        prm.rows = sh.rows;
        prm.n_rt = p->n_rt;
        prm.timeout_ns = ctx->timeout_ns;
        prm.stall = ctx->stall_test;
        const bool prof = p->profile && p->ev_used + 2 <= p->ev.size();
        if (prof) cudaEventRecord(p->ev[p->ev_used], st);
        cudaError_t e;
        if (p->pair && sh.hd == 256) {
            e = sh.quant == PA_CUDA_Q8_0 ? launch_prefill_pair<1, 1, 256>(p, nj, tq, prm, st)
                                         : launch_prefill_pair<2, 1, 256>(p, nj, tq, prm, st);
        } else if (p->pair) {
            if (sh.quant == PA_CUDA_Q8_0)
                e = p->nt == 2 ? launch_prefill_pair<1, 2, 128>(p, nj, tq, prm, st) : launch_prefill_pair<1, 1, 128>(p, nj, tq, prm, st);
            else
                e = p->nt == 2 ? launch_prefill_pair<2, 2, 128>(p, nj, tq, prm, st) : launch_prefill_pair<2, 1, 128>(p, nj, tq, prm, st);
        } else if (sh.hd == 256) {   // one Q tile of 128 rows per CTA
            e = sh.quant == PA_CUDA_Q8_0 ? launch_prefill<1, 1, 256>(p, nj, tq, prm, st)
                                         : launch_prefill<2, 1, 256>(p, nj, tq, prm, st);
        } else if (sh.quant == PA_CUDA_Q8_0) {
            e = p->nt == 2 ? launch_prefill<1, 2>(p, nj, tq, prm, st) : launch_prefill<1, 1>(p, nj, tq, prm, st);
        } else {
            e = p->nt == 2 ? launch_prefill<2, 2>(p, nj, tq, prm, st) : launch_prefill<2, 1>(p, nj, tq, prm, st);
        }
        if (e != cudaSuccess) return cuda_fail(ctx, e, "prefill kernel launch");
        if (prof) {
            cudaEventRecord(p->ev[p->ev_used + 1], st);
            p->ev_used += 2;
        }
        ctx->launches++;
    } else if (nj > 0) {
        pa::dec::Params prm{};
        prm.jobs = p->d_jobs + j0;
        prm.Qs = Qs;
        prm.Op = p->d_op;
        prm.Mp = p->d_mp;
        prm.Lp = p->d_lp;
        prm.status = ctx->d_status;
        prm.rs = sh.rs;
        prm.hb = sh.hb;
        prm.nkv = sh.nkv;
        prm.rows = sh.rows;
        prm.hg = p->hg;
        prm.rgc = p->rgc;
        prm.n_rg = p->n_rg;
        prm.row = p->row;
        prm.gs = p->gs;
        prm.n_jobs = nj;
        prm.n_consumers = p->n_consumers;
        prm.timeout_ns = ctx->timeout_ns;
        prm.stall = ctx->stall_test;
        const bool prof = p->profile && p->ev_used + 2 <= p->ev.size();
        if (prof) cudaEventRecord(p->ev[p->ev_used], st);
        cudaError_t e;
        e = launch_decode_any(p, nj, prm, st, sh.hd, sh.quant);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "decode kernel launch");
        if (prof) {
            cudaEventRecord(p->ev[p->ev_used + 1], st);
            p->ev_used += 2;
        }
        ctx->launches++;
    }
    return PA_CUDA_OK;
}
int run_plan_sets(pa_cuda_plan *p, const uint16_t *Qs, float *O, float *m, float *l, cudaStream_t st, uint32_t s0,
                  uint32_t s1) {
    pa_cuda_ctx *ctx = p->ctx;
    const pa_cuda_shape &sh = p->sh;
    int rc = run_attention_sets(p, Qs, st, s0, s1);
    if (rc) return rc;
    pa::mrg::Params mp{};
    mp.Op = p->d_op;
    mp.Mp = p->d_mp;
    mp.Lp = p->d_lp;
    mp.c_range = p->d_crange + s0;
    mp.n_parts = p->n_slots;
    mp.op_stride = (uint64_t) sh.nkv * sh.rows * sh.hd;
    mp.ml_stride = (uint64_t) sh.nkv * sh.rows;
    mp.set_rows = 0;
    mp.O = O;
    mp.M = m;
    mp.L = l;
    mp.rows_per_set = (uint64_t) sh.nkv * sh.rows;
    mp.n_sets = s1 - s0;
    mp.fold = 0;
    cudaError_t e = sh.hd == 128 ? launch_merge<128>(mp, st, ctx->n_sm) : launch_merge<256>(mp, st, ctx->n_sm);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "merge kernel launch");
    ctx->launches++;
    return PA_CUDA_OK;
}
int run_plan(pa_cuda_plan *p, const uint16_t *Qs, float *O, float *m, float *l, cudaStream_t st) {
    return run_plan_sets(p, Qs, O, m, l, st, 0, p->n_sets);
}

template <class T>
int ensure_dev(pa_cuda_ctx *ctx, T *&ptr, size_t &cap, size_t bytes) {
    if (cap >= bytes && ptr) return PA_CUDA_OK;
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    cap = 0;
    cudaError_t e = cudaMalloc((void **) &ptr, std::max<size_t>(bytes, 256));
    if (e != cudaSuccess) return fail(ctx, PA_CUDA_ENOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
    cap = std::max<size_t>(bytes, 256);
    return PA_CUDA_OK;
}
template <class T>
int ensure_host(pa_cuda_ctx *ctx, T *&ptr, size_t &cap, size_t bytes) {
    if (cap >= bytes && ptr) return PA_CUDA_OK;
    if (ptr) cudaFreeHost(ptr);
    ptr = nullptr;
    cap = 0;
    cudaError_t e = cudaMallocHost((void **) &ptr, std::max<size_t>(bytes, 256));
    if (e != cudaSuccess) return fail(ctx, PA_CUDA_ENOMEM, std::string("cudaMallocHost: ") + cudaGetErrorString(e));
    cap = std::max<size_t>(bytes, 256);
    return PA_CUDA_OK;
}

// NCCL, opened on first use (libnccl.so.2: the copy already in the process, e.g. torch's, else the system's), so the
// library has no link-time dependency on it and callers that never shard never load it
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*comm_abort)(ncclComm_t);
    ncclResult_t (*comm_async_error)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*comm_count)(const ncclComm_t, int *);
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int *);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*group_start)();
    ncclResult_t (*group_end)();
    const char *(*get_error_string)(ncclResult_t);
};
const NcclApi *nccl_api() {
    static const NcclApi *api = []() -> const NcclApi * {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) return nullptr;
        static NcclApi a;
        a.get_unique_id = (decltype(a.get_unique_id)) dlsym(h, "ncclGetUniqueId");
        a.comm_init_rank = (decltype(a.comm_init_rank)) dlsym(h, "ncclCommInitRank");
        a.comm_destroy = (decltype(a.comm_destroy)) dlsym(h, "ncclCommDestroy");
        a.comm_abort = (decltype(a.comm_abort)) dlsym(h, "ncclCommAbort");
        a.comm_async_error = (decltype(a.comm_async_error)) dlsym(h, "ncclCommGetAsyncError");
        a.comm_count = (decltype(a.comm_count)) dlsym(h, "ncclCommCount");
        a.comm_user_rank = (decltype(a.comm_user_rank)) dlsym(h, "ncclCommUserRank");
        a.all_gather = (decltype(a.all_gather)) dlsym(h, "ncclAllGather");
        a.all_reduce = (decltype(a.all_reduce)) dlsym(h, "ncclAllReduce");
        a.group_start = (decltype(a.group_start)) dlsym(h, "ncclGroupStart");
        a.group_end = (decltype(a.group_end)) dlsym(h, "ncclGroupEnd");
        a.get_error_string = (decltype(a.get_error_string)) dlsym(h, "ncclGetErrorString");
        if (!a.get_unique_id || !a.comm_init_rank || !a.comm_destroy || !a.comm_abort || !a.comm_async_error ||
            !a.comm_count || !a.comm_user_rank || !a.all_gather || !a.all_reduce || !a.group_start || !a.group_end ||
            !a.get_error_string)
            return nullptr;
        return &a;
    }();
    return api;
}
int nccl_fail(pa_cuda_ctx *ctx, const NcclApi *api, ncclResult_t r, const char *what) {
    return fail(ctx, PA_CUDA_ENCCL, std::string(what) + ": " + api->get_error_string(r));
}

// a shard communicator: NCCL's, plus whether it was aborted (after which NCCL has freed it)
struct ShardComm {
    ncclComm_t nc = nullptr;
    int rank = 0, world = 1, device = 0;
    bool dead = false;
    // peer-store exchange: every rank holds one buffer, mapped into every other rank with CUDA IPC: flags
    // [world source ranks][blocks_cap] (u64: the call number a source's block last published), then the receive area
    // [2 halves by call parity][world source ranks][cap floats]
    int p2p_state = 0;                        // 0 not set up, 1 ready, -1 unavailable on some rank (all fall back)
    uint8_t *p2p_buf = nullptr;
    size_t p2p_cap = 0, p2p_blocks = 0, p2p_head = 0;   // floats of a part, blocks of a call, bytes of the flags
    std::vector<uint8_t *> p2p_peer;          // each rank's buffer as mapped here (this rank's own: p2p_buf)
    float **d_push = nullptr;                 // device [world]: rank r's receive area, slot of this rank, half 0
    unsigned long long **d_pflag = nullptr;   // device [world]: rank r's flags of source = this rank
    unsigned long long p2p_calls = 0;         // peer-store calls so far (the epoch of the next is p2p_calls + 1)
};
constexpr uint32_t kSetupWaitMs = 60000;   // bound on the set-up collectives of the peer-store exchange
// exchange choices by size: the two-all-reduce exchange from this many bytes of one rank's partial (with more than 2
// ranks), and set groups whose exchange overlaps the next group's kernels from this many
constexpr size_t kShardReduceBytes = 8u << 20;
constexpr size_t kShardGroupBytes = 64u << 20;
constexpr uint32_t kShardGroups = 8;

// Wait for the work queued on st, polling the stream and NCCL's asynchronous error; on an NCCL error, or when the bound
// passes (a rank that left or stopped answering leaves the collective waiting for it), abort the communicator so that
// its kernels return and the stream drains, and report it. The communicator is unusable afterwards.
int shard_wait(pa_cuda_ctx *ctx, const NcclApi *api, ShardComm *sc, cudaStream_t st, uint32_t timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    auto elapsed_ms = [&]() {
        return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    };
    int code = PA_CUDA_OK;
    std::string why;
    for (;;) {
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) return PA_CUDA_OK;
        if (q != cudaErrorNotReady) return cuda_fail(ctx, q, "stream query");
        ncclResult_t ar = ncclSuccess;
        if (sc->dead) { code = PA_CUDA_ENCCL; why = "the communicator was aborted earlier"; break; }
        if (api->comm_async_error(sc->nc, &ar) == ncclSuccess && ar != ncclSuccess && ar != ncclInProgress) {
            code = PA_CUDA_ENCCL;
            why = std::string("NCCL asynchronous error: ") + api->get_error_string(ar);
            break;
        }
        if (timeout_ms && elapsed_ms() > timeout_ms) {
            code = PA_CUDA_ETIMEOUT;
            why = "the shard exchange did not finish within " + std::to_string(timeout_ms) + " ms (a rank left or stalled)";
            break;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    if (!sc->dead) {
        api->comm_abort(sc->nc);   // its kernels in flight return; the communicator's resources are released
        sc->dead = true;
    }
    // the stream drains once the aborted collectives have returned (bounded)
    const auto t1 = std::chrono::steady_clock::now();
    while (cudaStreamQuery(st) == cudaErrorNotReady &&
           std::chrono::steady_clock::now() - t1 < std::chrono::seconds(10))
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    cudaGetLastError();
    return fail(ctx, code, why + "; communicator aborted");
}

void p2p_release(ShardComm *sc) {
    cudaSetDevice(sc->device);
    for (int r = 0; r < (int) sc->p2p_peer.size(); r++)
        if (r != sc->rank && sc->p2p_peer[r]) cudaIpcCloseMemHandle(sc->p2p_peer[r]);
    sc->p2p_peer.clear();
    if (sc->p2p_buf) cudaFree(sc->p2p_buf);
    if (sc->d_push) cudaFree(sc->d_push);
    if (sc->d_pflag) cudaFree(sc->d_pflag);
    sc->p2p_buf = nullptr;
    sc->d_push = nullptr;
    sc->d_pflag = nullptr;
    sc->p2p_cap = sc->p2p_blocks = sc->p2p_head = 0;
    cudaGetLastError();
}

// every rank's answer to "did this step work here" (an all-gather of one byte each); the ranks act on the same answer
bool all_ranks_ok(pa_cuda_ctx *ctx, const NcclApi *api, ShardComm *sc, bool ok, cudaStream_t st) {
    uint8_t *d = nullptr;
    std::vector<uint8_t> h((size_t) sc->world, 0);
    bool all = cudaMalloc((void **) &d, (size_t) sc->world) == cudaSuccess;
    const uint8_t mine = ok ? 1 : 0;
    if (all) all = cudaMemcpy(d + sc->rank, &mine, 1, cudaMemcpyHostToDevice) == cudaSuccess;
    // the all-gather runs on every rank whatever happened here, so that no rank waits for another forever
    const ncclResult_t r = api->all_gather(all ? d + sc->rank : nullptr, d, 1, ncclUint8, sc->nc, st);
    all = all && r == ncclSuccess && shard_wait(ctx, api, sc, st, kSetupWaitMs) == PA_CUDA_OK &&
          cudaMemcpy(h.data(), d, (size_t) sc->world, cudaMemcpyDeviceToHost) == cudaSuccess;
    if (d) cudaFree(d);
    for (int i = 0; all && i < sc->world; i++) all = h[(size_t) i] == 1;
    return all;
}

// Sets up (collectively: every rank calls it at the same point) the peer-store buffers for parts of `part` floats: each
// rank allocates its buffer, the IPC handles go round with one all-gather, and each rank maps the others'. If any
// rank fails at any step every rank drops the exchange (state -1) and the shard call uses NCCL instead.
void p2p_setup(pa_cuda_ctx *ctx, const NcclApi *api, ShardComm *sc, size_t part, size_t blocks, cudaStream_t st) {
    if (sc->p2p_state == 1 && sc->p2p_cap >= part && sc->p2p_blocks >= blocks) return;
    if (sc->p2p_state == -1) return;
    p2p_release(sc);
    const int W = sc->world;
    const size_t head = ((size_t) W * blocks * 8 + 255) / 256 * 256;
    const size_t bytes = head + 2 * (size_t) W * part * sizeof(float);
    bool ok = cudaMalloc((void **) &sc->p2p_buf, bytes) == cudaSuccess &&
              cudaMemset(sc->p2p_buf, 0, head) == cudaSuccess;
    cudaIpcMemHandle_t mine{};
    if (ok) ok = cudaIpcGetMemHandle(&mine, sc->p2p_buf) == cudaSuccess;
    // the handles (plus a success byte) of every rank
    constexpr size_t HB = sizeof(cudaIpcMemHandle_t) + 8;
    uint8_t *d = nullptr;
    std::vector<uint8_t> h((size_t) W * HB, 0);
    const bool dev_ok = cudaMalloc((void **) &d, (size_t) W * HB) == cudaSuccess;
    if (dev_ok) {
        std::vector<uint8_t> me(HB, 0);
        memcpy(me.data(), &mine, sizeof mine);
        me[sizeof mine] = ok ? 1 : 0;
        cudaMemcpy(d + (size_t) sc->rank * HB, me.data(), HB, cudaMemcpyHostToDevice);
    }
    const ncclResult_t r = api->all_gather(dev_ok ? d + (size_t) sc->rank * HB : nullptr, d, HB, ncclUint8, sc->nc, st);
    ok = ok && dev_ok && r == ncclSuccess && shard_wait(ctx, api, sc, st, kSetupWaitMs) == PA_CUDA_OK &&
         cudaMemcpy(h.data(), d, h.size(), cudaMemcpyDeviceToHost) == cudaSuccess;
    if (d) cudaFree(d);
    for (int i = 0; ok && i < W; i++) ok = h[(size_t) i * HB + sizeof mine] == 1;
    // map every other rank's buffer
    sc->p2p_peer.assign((size_t) W, nullptr);
    sc->p2p_peer[(size_t) sc->rank] = sc->p2p_buf;
    for (int i = 0; ok && i < W; i++) {
        if (i == sc->rank) continue;
        cudaIpcMemHandle_t hi;
        memcpy(&hi, h.data() + (size_t) i * HB, sizeof hi);
        void *ptr = nullptr;
        ok = cudaIpcOpenMemHandle(&ptr, hi, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        sc->p2p_peer[(size_t) i] = (uint8_t *) ptr;
    }
    cudaGetLastError();
    // device tables: where this rank's part goes in each rank, and its counter there
    if (ok) {
        std::vector<float *> push((size_t) W);
        std::vector<unsigned long long *> flag((size_t) W);
        for (int i = 0; i < W; i++) {
            push[(size_t) i] = (float *) (sc->p2p_peer[(size_t) i] + head) + (size_t) sc->rank * part;
            flag[(size_t) i] = (unsigned long long *) sc->p2p_peer[(size_t) i] + (size_t) sc->rank * blocks;
        }
        ok = cudaMalloc((void **) &sc->d_push, W * sizeof(float *)) == cudaSuccess &&
             cudaMalloc((void **) &sc->d_pflag, W * sizeof(unsigned long long *)) == cudaSuccess &&
             cudaMemcpy(sc->d_push, push.data(), W * sizeof(float *), cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(sc->d_pflag, flag.data(), W * sizeof(unsigned long long *), cudaMemcpyHostToDevice) == cudaSuccess;
    }
    // the same decision on every rank
    ok = all_ranks_ok(ctx, api, sc, ok, st);
    if (!ok) {
        p2p_release(sc);
        sc->p2p_state = -1;
        return;
    }
    sc->p2p_state = 1;
    sc->p2p_cap = part;
    sc->p2p_blocks = blocks;
    sc->p2p_head = head;
    sc->p2p_calls = 0;
}

}  // namespace

// ====================================================================================================== C ABI
extern "C" {

int pa_cuda_abi_version(void) { return PA_CUDA_ABI_VERSION; }

int pa_cuda_available(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return 0;
    }
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
    if (major != 10) return 0;
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, pa::dec::decode_kernel<128, 1, 8>) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return 1;
}

int pa_cuda_create(int device, pa_cuda_ctx **out) {
    if (!out) return PA_CUDA_EINVAL;
    *out = nullptr;
    auto *ctx = new pa_cuda_ctx();
    ctx->device = device;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) { delete ctx; return PA_CUDA_ECUDA; }
    cudaDeviceGetAttribute(&ctx->n_sm, cudaDevAttrMultiProcessorCount, device);
    if ((e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaMalloc((void **) &ctx->d_status, 16)) != cudaSuccess ||
        (e = cudaMallocHost((void **) &ctx->h_status, 16)) != cudaSuccess ||
        (e = cudaMemset(ctx->d_status, 0, 16)) != cudaSuccess || (e = cudaEventCreate(&ctx->ev_begin)) != cudaSuccess ||
        (e = cudaEventCreate(&ctx->ev_end)) != cudaSuccess) {
        pa_cuda_destroy(ctx);
        return PA_CUDA_ECUDA;
    }
    *out = ctx;
    return PA_CUDA_OK;
}

void pa_cuda_destroy(pa_cuda_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (auto &e : ctx->eng_cache) {
        if (e.graph) cudaGraphExecDestroy(e.graph);
        if (e.plan) pa_cuda_plan_destroy(e.plan);
    }
    if (ctx->h_q) cudaFreeHost(ctx->h_q);
    if (ctx->h_out) cudaFreeHost(ctx->h_out);
    if (ctx->d_q) cudaFree(ctx->d_q);
    if (ctx->d_out) cudaFree(ctx->d_out);
    if (ctx->ev_begin) cudaEventDestroy(ctx->ev_begin);
    if (ctx->ev_end) cudaEventDestroy(ctx->ev_end);
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->h_status) cudaFreeHost(ctx->h_status);
    if (ctx->d_shard) cudaFree(ctx->d_shard);
    if (ctx->d_gathered) cudaFree(ctx->d_gathered);
    for (auto e : ctx->xev) cudaEventDestroy(e);
    if (ctx->xstream) cudaStreamDestroy(ctx->xstream);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

const char *pa_cuda_last_error(const pa_cuda_ctx *ctx) { return ctx ? ctx->err.c_str() : "no context"; }

void pa_cuda_set_timeout_ns(pa_cuda_ctx *ctx, uint64_t ns) {
    if (ctx) ctx->timeout_ns = ns;
}

uint64_t pa_cuda_launch_count(const pa_cuda_ctx *ctx) { return ctx ? ctx->launches : 0; }

void pa_cuda_set_kernel(pa_cuda_ctx *ctx, int which) {
    if (ctx) ctx->kernel_choice = which;
}

void pa_cuda_set_qk_domain(pa_cuda_ctx *ctx, int domain) {
    if (ctx) ctx->qk_domain = domain == PA_CUDA_QK_INT8 ? PA_CUDA_QK_INT8 : PA_CUDA_QK_F16;
}

void pa_cuda_set_stall_test(pa_cuda_ctx *ctx, int on) {
    if (ctx) ctx->stall_test = on ? 1 : 0;
}

int pa_cuda_status(pa_cuda_ctx *ctx, void *stream) {
    if (!ctx) return PA_CUDA_EINVAL;
    cudaStream_t st = pick(ctx, stream);
    // the read and the clear stay on the caller's stream (no legacy-stream copy that would wait for every blocking
    // stream of the process, or fail under another thread's global-mode capture)
    PA_CK(cudaSetDevice(ctx->device), "cudaSetDevice");
    PA_CK(cudaMemcpyAsync(ctx->h_status, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, st), "status read");
    PA_CK(cudaStreamSynchronize(st), "stream synchronize");
    const int h = *ctx->h_status;
    if (h != pa::ST_OK) {
        PA_CK(cudaMemsetAsync(ctx->d_status, 0, sizeof h, st), "status clear");
        PA_CK(cudaStreamSynchronize(st), "stream synchronize");
        return fail(ctx, PA_CUDA_ETIMEOUT, "a kernel gave up a bounded wait (code " + std::to_string(h) + ")");
    }
    return PA_CUDA_OK;
}

int pa_cuda_plan_create(pa_cuda_ctx *ctx, const pa_cuda_shape *shape, uint32_t n_sets, const pa_cuda_seg *segs,
                        uint32_t n_segs, uint32_t chunk_keys, pa_cuda_plan **out) {
    if (!ctx || !out) return PA_CUDA_EINVAL;
    *out = nullptr;
    int rc = check_shape(ctx, shape);
    if (rc) return rc;
    if (n_segs && !segs) return fail(ctx, PA_CUDA_EINVAL, "segs is null");
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, PA_CUDA_ECUDA, "cudaSetDevice");
    auto *p = new pa_cuda_plan();
    p->ctx = ctx;
    p->sh = *shape;
    p->n_sets = n_sets;
    if ((rc = plan_decode_shape(ctx, p))) { delete p; return rc; }
    if (ctx->qk_domain == PA_CUDA_QK_INT8) {
        // the int8-domain QK (sme_attn.c:465-508) reads Q8_0 bytes and runs on the split-K kernel only
        if (shape->quant != PA_CUDA_Q8_0 || ctx->kernel_choice >= 2) {
            delete p;
            return fail(ctx, PA_CUDA_EUNSUPPORTED, "the int8-domain QK needs Q8_0 rows and the split-K kernel");
        }
        p->qk_i8 = true;
    }
    // the tcgen05 kernel takes calls with many query rows per KV head (prefill, ATTN_BIG, long verify batches), the
    // split-K kernel the decode-sized ones (as the reference engine switches kernels by rows, pa-metal.mm:818-835)
    // (hd 256, the reference server's wire geometry: one 128-row tile per CTA up to kSingle256MaxRows rows per KV head,
    // CTA pairs above)
    const bool tc_ok = (shape->hd == 128 || shape->hd == 256) && shape->quant != PA_CUDA_F16 && encode_fn() != nullptr;
    const uint32_t min_rows = shape->hd == 128 ? kPrefillMinRows128 : kPrefillMinRows256;
    p->prefill = tc_ok && !p->qk_i8 && (ctx->kernel_choice >= 2 || (ctx->kernel_choice == 0 && shape->rows >= min_rows));
    if (ctx->kernel_choice >= 2 && !tc_ok) {
        delete p;
        return fail(ctx, PA_CUDA_EUNSUPPORTED,
                    "tcgen05 kernels need quantised (Q8_0 / Q4_0) rows and hd 128 or 256");
    }
    if (p->prefill) {
        // PA_CUDA_TC_TILES=1|2: Q tiles of 128 rows per CTA (default: 2 when there are more than 128 rows)
        static const int tiles_env = getenv("PA_CUDA_TC_TILES") ? atoi(getenv("PA_CUDA_TC_TILES")) : 0;
        // CTA pairs (2-SM MMAs, half of each K/V block dequantised per SM) from kPairMinRows rows per KV head
        p->pair = ctx->kernel_choice == 3 ||
                  (ctx->kernel_choice == 0 && shape->rows >= (shape->hd == 256 ? kSingle256MaxRows + 1 : kPairMinRows));
        const uint32_t tile_rows = (uint32_t) pa::pre::BM * (p->pair ? 2u : 1u);
        p->nt = shape->hd == 256 ? 1 : (tiles_env == 1 || tiles_env == 2) ? tiles_env : (shape->rows > tile_rows ? 2 : 1);
        p->n_rt = (shape->rows + tile_rows * p->nt - 1) / (tile_rows * p->nt);
        p->grid_y = shape->nkv * p->n_rt;
    }

    uint64_t total = 0;
    for (uint32_t i = 0; i < n_segs; i++) {
        if (segs[i].set >= n_sets) { delete p; return fail(ctx, PA_CUDA_EINVAL, "segment set index >= n_sets"); }
        if (segs[i].nk && (((uintptr_t) segs[i].k | (uintptr_t) segs[i].v) & 15)) {
            delete p;
            return fail(ctx, PA_CUDA_EINVAL, "segment K/V pointers must be 16-byte aligned");
        }
        total += segs[i].nk;
    }
    uint32_t chunk = chunk_keys;
    if (chunk == 0 && p->prefill) {
        // The job size that minimises waves x (keys per job + kPrefillJobOverhead), waves counting the CTAs of all jobs
        // (every row group and KV head of a job; two per cluster) over one CTA per SM: a small call (the server's
        // 8-token ATTN over 32k keys) gets about one wave of longer jobs instead of many short CTAs that each pay the
        // set-up (TMEM, barriers, Q tiles, the ring's first stages); config 2 keeps a 65,536-key segment per job and
        // the config-3 verify batch two jobs per 196,608-key layer (7 waves of 1,024 CTAs).
        const uint64_t ctas_per_job = (uint64_t) p->grid_y * (p->pair ? 2 : 1);
        uint64_t best = ~0ull;
        for (uint32_t c = 512; c <= 262144; c += 512) {
            uint64_t jobs = 0, cmax = 0;
            for (uint32_t i = 0; i < n_segs; i++) {
                const uint32_t nk = segs[i].nk;
                if (!nk) continue;
                const uint32_t nj = (nk + c - 1) / c, cj = ((nk + nj - 1) / nj + 63) / 64 * 64;
                jobs += (nk + cj - 1) / cj;
                cmax = std::max<uint64_t>(cmax, cj);
            }
            const uint64_t waves = (jobs * ctas_per_job + ctx->n_sm - 1) / ctx->n_sm;
            const uint64_t cost = waves * (cmax + kPrefillJobOverhead);
            if (cost <= best) { best = cost; chunk = c; }
        }
        if (!chunk) chunk = 1024;
    } else if (chunk == 0) {
        // The job size that minimises the modelled time: waves x (keys per job + kDecodeJobOverhead). Waves count the
        // CTAs that fit all SMs at once.
        const uint32_t slots = (uint32_t) ctx->n_sm * (uint32_t) decode_ctas_per_sm(p);
        const uint32_t overhead = kDecodeJobOverhead;
        uint64_t best = ~0ull;
        for (uint32_t c = 128; c <= 16384; c += 64) {
            uint64_t jobs = 0, cmax = 0;
            for (uint32_t i = 0; i < n_segs; i++) {
                const uint32_t nk = segs[i].nk;
                if (!nk) continue;
                const uint32_t nj = (nk + c - 1) / c, cj = ((nk + nj - 1) / nj + 63) / 64 * 64;
                jobs += (nk + cj - 1) / cj;
                cmax = std::max<uint64_t>(cmax, cj);
            }
            const uint64_t waves = (jobs * p->grid_y + slots - 1) / slots;
            const uint64_t cost = waves * (cmax + overhead);
            if (cost <= best) { best = cost; chunk = c; }
        }
        if (!chunk) chunk = 128;
    }
    chunk = (chunk + 63) / 64 * 64;

    // jobs grouped by set, so that the slots of a set are contiguous
    std::vector<pa::dec::Job> jobs;
    std::vector<uint32_t> crange(n_sets + 1, 0);
    for (uint32_t s = 0; s < n_sets; s++) {
        crange[s] = (uint32_t) jobs.size();
        for (uint32_t i = 0; i < n_segs; i++) {
            if (segs[i].set != s || segs[i].nk == 0) continue;
            const uint32_t nk = segs[i].nk;
            const uint32_t nj = (nk + chunk - 1) / chunk;
            const uint32_t cj = ((nk + nj - 1) / nj + 63) / 64 * 64;   // equal chunks of whole stages / blocks
            for (uint32_t k0 = 0; k0 < nk; k0 += cj) {
                pa::dec::Job j;
                j.k = segs[i].k;
                j.v = segs[i].v;
                j.key0 = k0;
                j.nk = std::min(cj, nk - k0);
                j.set = s;
                j.slot = (uint32_t) jobs.size();
                j.seg = i;
                j.pad_ = 0;
                jobs.push_back(j);
            }
        }
    }
    crange[n_sets] = (uint32_t) jobs.size();
    p->crange = crange;
    p->n_jobs = p->n_slots = (uint32_t) jobs.size();
    if (p->n_jobs > 0 && p->grid_y > 65535) { delete p; return fail(ctx, PA_CUDA_EUNSUPPORTED, "too many head/row groups"); }

    const size_t rows_all = (size_t) shape->nkv * shape->rows;
    const size_t op_b = (size_t) p->n_slots * rows_all * shape->hd * 4, ml_b = (size_t) p->n_slots * rows_all * 4;
    p->scratch = op_b + 2 * ml_b;
    cudaError_t e = cudaSuccess;
    if (p->n_jobs) {
        if ((e = cudaMalloc((void **) &p->d_jobs, jobs.size() * sizeof(pa::dec::Job))) == cudaSuccess &&
            (e = cudaMalloc((void **) &p->d_op, op_b)) == cudaSuccess &&
            (e = cudaMalloc((void **) &p->d_mp, ml_b)) == cudaSuccess &&
            (e = cudaMalloc((void **) &p->d_lp, ml_b)) == cudaSuccess)
            e = cudaMemcpy(p->d_jobs, jobs.data(), jobs.size() * sizeof(pa::dec::Job), cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess && (e = cudaMalloc((void **) &p->d_crange, crange.size() * 4)) == cudaSuccess)
        e = cudaMemcpy(p->d_crange, crange.data(), crange.size() * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && p->prefill && n_segs) {
        std::vector<CUtensorMap> maps(2 * (size_t) n_segs);
        const uint32_t rawb = (uint32_t) pa::pre::raw_row_bytes((int) shape->quant, (int) shape->hd);
        for (uint32_t i = 0; i < n_segs; i++) {
            if (!segs[i].nk) continue;
            // a CTA of a pair loads half of each block's K rows and all of its V rows
            const uint32_t kbox = p->pair ? (uint32_t) pa::pre::BN / 2 : (uint32_t) pa::pre::BN;
            if (!map_rows(&maps[2 * i], segs[i].k, shape->rs, segs[i].nk, rawb, kbox) ||
                !map_rows(&maps[2 * i + 1], segs[i].v, shape->rs, segs[i].nk, rawb, (uint32_t) pa::pre::BN)) {
                pa_cuda_plan_destroy(p);
                return fail(ctx, PA_CUDA_ECUDA, "cuTensorMapEncodeTiled (K/V rows) failed");
            }
        }
        if ((e = cudaMalloc((void **) &p->d_maps, maps.size() * sizeof(CUtensorMap))) == cudaSuccess)
            e = cudaMemcpy(p->d_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        pa_cuda_plan_destroy(p);
        return fail(ctx, PA_CUDA_ENOMEM, std::string("plan allocation: ") + cudaGetErrorString(e));
    }
    *out = p;
    return PA_CUDA_OK;
}

size_t pa_cuda_plan_scratch_bytes(const pa_cuda_plan *p) { return p ? p->scratch : 0; }
uint32_t pa_cuda_plan_jobs(const pa_cuda_plan *p) { return p ? p->n_jobs : 0; }
uint32_t pa_cuda_plan_launches(const pa_cuda_plan *p) { return p ? (p->n_jobs ? 2u : 1u) : 0u; }

const char *pa_cuda_plan_kernel(const pa_cuda_plan *p) {
    if (!p) return "";
    const uint32_t q = p->sh.quant;
    if (p->prefill) {
        static const char *names[4][2][2] = {
            {{"pa::pre::prefill_kernel<1,1,128>", "pa::pre::prefill_kernel<1,2,128>"},
             {"pa::pre::prefill_kernel<2,1,128>", "pa::pre::prefill_kernel<2,2,128>"}},
            {{"pa::pre::prefill_pair_kernel<1,1,128>", "pa::pre::prefill_pair_kernel<1,2,128>"},
             {"pa::pre::prefill_pair_kernel<2,1,128>", "pa::pre::prefill_pair_kernel<2,2,128>"}},
            {{"pa::pre::prefill_pair_kernel<1,1,256>", "pa::pre::prefill_pair_kernel<1,1,256>"},
             {"pa::pre::prefill_pair_kernel<2,1,256>", "pa::pre::prefill_pair_kernel<2,1,256>"}},
            {{"pa::pre::prefill_kernel<1,1,256>", "pa::pre::prefill_kernel<1,1,256>"},
             {"pa::pre::prefill_kernel<2,1,256>", "pa::pre::prefill_kernel<2,1,256>"}}};
        const int k = !p->pair ? (p->sh.hd == 256 ? 3 : 0) : p->sh.hd == 256 ? 2 : 1;
        return names[k][q == PA_CUDA_Q8_0 ? 0 : 1][p->nt == 2 ? 1 : 0];
    }
    static const char *dec[3][4] = {
        {"pa::dec::decode_kernel<128,0,8>", "pa::dec::decode_kernel<128,1,8>", "pa::dec::decode_kernel<128,2,8>",
         "pa::dec::decode_kernel<128,3,8>"},
        {"pa::dec::decode_kernel<256,0,8>", "pa::dec::decode_kernel<256,1,8>", "pa::dec::decode_kernel<256,2,8>",
         "pa::dec::decode_kernel<256,3,8>"},
        {"pa::dec::decode_kernel<256,0,4>", "pa::dec::decode_kernel<256,1,4>", "pa::dec::decode_kernel<256,2,4>",
         "pa::dec::decode_kernel<256,3,4>"}};
    return dec[p->sh.hd == 128 ? 0 : p->w == 4 ? 2 : 1][p->qk_i8 ? 3 : q <= 2 ? q : 0];
}

int pa_cuda_plan_run(pa_cuda_plan *p, const uint16_t *Qs, float *O, float *m, float *l, void *stream) {
    if (!p) return PA_CUDA_EINVAL;
    pa_cuda_ctx *ctx = p->ctx;
    if (!O || !m || !l || (p->n_jobs && !Qs)) return fail(ctx, PA_CUDA_EINVAL, "null Q/O/m/l");
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, PA_CUDA_ECUDA, "cudaSetDevice");
    return run_plan(p, Qs, O, m, l, pick(ctx, stream));
}

int pa_cuda_plan_profile(pa_cuda_plan *p, uint32_t max_runs) {
    if (!p) return PA_CUDA_EINVAL;
    pa_cuda_ctx *ctx = p->ctx;
    cudaSetDevice(ctx->device);
    for (auto e : p->ev) cudaEventDestroy(e);
    p->ev.clear();
    p->ev_used = 0;
    p->profile = max_runs > 0;
    for (uint32_t i = 0; i < 2 * max_runs; i++) {
        cudaEvent_t e;
        PA_CK(cudaEventCreate(&e), "event create");
        p->ev.push_back(e);
    }
    return PA_CUDA_OK;
}

int pa_cuda_plan_kernel_ms(pa_cuda_plan *p, double *total_ms, uint32_t *n_runs) {
    if (!p || !total_ms || !n_runs) return PA_CUDA_EINVAL;
    pa_cuda_ctx *ctx = p->ctx;
    double t = 0;
    for (uint32_t i = 0; i + 1 < p->ev_used; i += 2) {
        PA_CK(cudaEventSynchronize(p->ev[i + 1]), "event synchronize");
        float ms = 0;
        PA_CK(cudaEventElapsedTime(&ms, p->ev[i], p->ev[i + 1]), "event elapsed");
        t += ms;
    }
    *total_ms = t;
    *n_runs = p->ev_used / 2;
    p->ev_used = 0;
    return PA_CUDA_OK;
}

void pa_cuda_plan_destroy(pa_cuda_plan *p) {
    if (!p) return;
    cudaSetDevice(p->ctx->device);
    for (auto e : p->ev) cudaEventDestroy(e);
    if (p->d_jobs) cudaFree(p->d_jobs);
    if (p->d_crange) cudaFree(p->d_crange);
    if (p->d_maps) cudaFree(p->d_maps);
    if (p->d_op) cudaFree(p->d_op);
    if (p->d_mp) cudaFree(p->d_mp);
    if (p->d_lp) cudaFree(p->d_lp);
    delete p;
}

int pa_cuda_attn(pa_cuda_ctx *ctx, const pa_cuda_shape *shape, const uint16_t *Qs, uint32_t n_sets,
                 const pa_cuda_seg *segs, uint32_t n_segs, float *O, float *m, float *l, void *stream) {
    pa_cuda_plan *p = nullptr;
    int rc = pa_cuda_plan_create(ctx, shape, n_sets, segs, n_segs, 0, &p);
    if (rc) return rc;
    rc = pa_cuda_plan_run(p, Qs, O, m, l, stream);
    cudaStreamSynchronize(pick(ctx, stream));
    pa_cuda_plan_destroy(p);
    return rc;
}

int pa_cuda_scale_q(pa_cuda_ctx *ctx, const float *Q, float scale, uint64_t n, uint16_t *Qs, void *stream) {
    if (!ctx || (n && (!Q || !Qs))) return fail(ctx, PA_CUDA_EINVAL, "null argument");
    if (n == 0) return PA_CUDA_OK;
    cudaSetDevice(ctx->device);
    const unsigned blocks = (unsigned) std::min<uint64_t>((n + 255) / 256, (uint64_t) ctx->n_sm * 8);
    pa::mrg::scale_q_kernel<<<blocks, 256, 0, pick(ctx, stream)>>>(Q, scale, n, Qs);
    PA_CK(cudaGetLastError(), "scale_q launch");
    ctx->launches++;
    return PA_CUDA_OK;
}

int pa_cuda_attn_partial(pa_cuda_ctx *ctx, const pa_cuda_shape *shape, const float *Q, float scale, const uint8_t *K,
                         const uint8_t *V, uint32_t nk, float *O, float *m, float *l, void *stream) {
    if (!ctx) return PA_CUDA_EINVAL;
    int rc = check_shape(ctx, shape);
    if (rc) return rc;
    const uint64_t n = (uint64_t) shape->nkv * shape->rows * shape->hd;
    uint16_t *Qs = nullptr;
    PA_CK(cudaMalloc((void **) &Qs, n * 2), "cudaMalloc Qs");
    rc = pa_cuda_scale_q(ctx, Q, scale, n, Qs, stream);
    if (!rc) {
        pa_cuda_seg seg{K, V, nk, 0};
        rc = pa_cuda_attn(ctx, shape, Qs, 1, &seg, nk ? 1u : 0u, O, m, l, stream);
    }
    cudaStreamSynchronize(pick(ctx, stream));
    cudaFree(Qs);
    if (!rc) rc = pa_cuda_status(ctx, stream);
    return rc;
}

int pa_cuda_plan_run_host(pa_cuda_plan *p, const uint16_t *Qs_host, float *O_host, float *m_host, float *l_host,
                          void *stream) {
    if (!p) return PA_CUDA_EINVAL;
    pa_cuda_ctx *ctx = p->ctx;
    if (!Qs_host || !O_host || !m_host || !l_host) return fail(ctx, PA_CUDA_EINVAL, "null host buffer");
    cudaSetDevice(ctx->device);
    cudaStream_t st = pick(ctx, stream);
    const size_t rows = (size_t) p->n_sets * p->sh.nkv * p->sh.rows;
    const size_t qb = rows * p->sh.hd * 2, ob = rows * p->sh.hd * 4, mb = rows * 4;
    int rc;
    if ((rc = ensure_dev(ctx, ctx->d_q, ctx->d_q_bytes, qb))) return rc;
    if ((rc = ensure_dev(ctx, ctx->d_out, ctx->d_out_bytes, ob + 2 * mb))) return rc;
    PA_CK(cudaMemcpyAsync(ctx->d_q, Qs_host, qb, cudaMemcpyHostToDevice, st), "Q to device");
    float *dO = ctx->d_out, *dm = (float *) ((char *) ctx->d_out + ob), *dl = dm + rows;
    if ((rc = run_plan(p, ctx->d_q, dO, dm, dl, st))) return rc;
    PA_CK(cudaMemcpyAsync(O_host, dO, ob, cudaMemcpyDeviceToHost, st), "O to host");
    PA_CK(cudaMemcpyAsync(m_host, dm, mb, cudaMemcpyDeviceToHost, st), "m to host");
    PA_CK(cudaMemcpyAsync(l_host, dl, mb, cudaMemcpyDeviceToHost, st), "l to host");
    PA_CK(cudaStreamSynchronize(st), "stream synchronize");
    return PA_CUDA_OK;
}

int pa_cuda_merge(pa_cuda_ctx *ctx, uint32_t hd, uint64_t rows, uint32_t n_parts, const float *Op, const float *mp,
                  const float *lp, float *O, float *m, float *l, int fold, void *stream) {
    if (!ctx) return PA_CUDA_EINVAL;
    if (hd != 128 && hd != 256) return fail(ctx, PA_CUDA_EUNSUPPORTED, "hd must be 128 or 256");
    if (!O || !m || !l || (n_parts && (!Op || !mp || !lp))) return fail(ctx, PA_CUDA_EINVAL, "null argument");
    cudaSetDevice(ctx->device);
    pa::mrg::Params prm{};
    prm.Op = Op;
    prm.Mp = mp;
    prm.Lp = lp;
    prm.c_range = nullptr;
    prm.n_parts = n_parts;
    prm.op_stride = rows * hd;
    prm.ml_stride = rows;
    prm.set_rows = 0;
    prm.O = O;
    prm.M = m;
    prm.L = l;
    prm.rows_per_set = rows;
    prm.n_sets = 1;
    prm.fold = fold ? 1 : 0;
    cudaError_t e = hd == 128 ? launch_merge<128>(prm, pick(ctx, stream), ctx->n_sm)
                              : launch_merge<256>(prm, pick(ctx, stream), ctx->n_sm);
    PA_CK(e, "merge launch");
    ctx->launches++;
    return PA_CUDA_OK;
}

int pa_cuda_merge_gathered(pa_cuda_ctx *ctx, uint32_t hd, uint64_t rows, uint32_t n_parts, const float *packed,
                           float *O, float *m, float *l, int fold, void *stream) {
    if (!ctx) return PA_CUDA_EINVAL;
    if (hd != 128 && hd != 256) return fail(ctx, PA_CUDA_EUNSUPPORTED, "hd must be 128 or 256");
    if (!O || !m || !l || (n_parts && !packed)) return fail(ctx, PA_CUDA_EINVAL, "null argument");
    cudaSetDevice(ctx->device);
    const uint64_t stride = rows * (hd + 2);
    pa::mrg::Params prm{};
    prm.Op = packed;
    prm.Mp = packed + rows * hd;
    prm.Lp = packed + rows * hd + rows;
    prm.c_range = nullptr;
    prm.n_parts = n_parts;
    prm.op_stride = stride;
    prm.ml_stride = stride;
    prm.set_rows = 0;
    prm.O = O;
    prm.M = m;
    prm.L = l;
    prm.rows_per_set = rows;
    prm.n_sets = 1;
    prm.fold = fold ? 1 : 0;
    cudaError_t e = hd == 128 ? launch_merge<128>(prm, pick(ctx, stream), ctx->n_sm)
                              : launch_merge<256>(prm, pick(ctx, stream), ctx->n_sm);
    PA_CK(e, "merge launch");
    ctx->launches++;
    return PA_CUDA_OK;
}

// ---------------------------------------------------------------------------------- position shards over NCCL
int pa_cuda_nccl_unique_id(void *id, size_t bytes) {
    const NcclApi *api = nccl_api();
    if (!api) return PA_CUDA_ENCCL;
    if (!id || bytes < sizeof(ncclUniqueId)) return PA_CUDA_EINVAL;
    ncclUniqueId u;
    if (api->get_unique_id(&u) != ncclSuccess) return PA_CUDA_ENCCL;
    memcpy(id, &u, sizeof u);
    return PA_CUDA_OK;
}

int pa_cuda_nccl_comm_create(pa_cuda_ctx *ctx, const void *id, int rank, int world, void **comm) {
    if (!ctx || !comm) return PA_CUDA_EINVAL;
    *comm = nullptr;
    if (!id || world < 1 || rank < 0 || rank >= world) return fail(ctx, PA_CUDA_EINVAL, "bad unique id, rank or world");
    const NcclApi *api = nccl_api();
    if (!api) return fail(ctx, PA_CUDA_ENCCL, "libnccl.so.2 could not be opened");
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, PA_CUDA_ECUDA, "cudaSetDevice");
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    ncclComm_t c = nullptr;
    const ncclResult_t r = api->comm_init_rank(&c, world, u, rank);
    if (r != ncclSuccess) return nccl_fail(ctx, api, r, "ncclCommInitRank");
    auto *sc = new ShardComm();
    sc->nc = c;
    sc->rank = rank;
    sc->world = world;
    sc->device = ctx->device;
    *comm = sc;
    return PA_CUDA_OK;
}

void pa_cuda_nccl_comm_destroy(void *comm) {
    auto *sc = (ShardComm *) comm;
    if (!sc) return;
    const NcclApi *api = nccl_api();
    // the peer-store buffers: mapped by the other ranks too, so destroy after they stopped calling (as with NCCL)
    cudaSetDevice(sc->device);
    cudaDeviceSynchronize();
    p2p_release(sc);
    if (api && sc->nc && !sc->dead) api->comm_destroy(sc->nc);
    delete sc;
}

void pa_cuda_set_shard_exchange(pa_cuda_ctx *ctx, int mode) {
    if (ctx) ctx->shard_exchange = (mode >= 0 && mode <= 3) ? mode : 0;
}
void pa_cuda_set_shard_groups(pa_cuda_ctx *ctx, int groups) {
    if (ctx) ctx->shard_groups = groups > 0 ? groups : 0;
}
void pa_cuda_set_shard_timeout_ms(pa_cuda_ctx *ctx, uint32_t ms) {
    if (ctx) ctx->shard_timeout_ms = ms;
}
void pa_cuda_shard_last(const pa_cuda_ctx *ctx, int *exchange, int *groups) {
    if (exchange) *exchange = ctx ? ctx->shard_last_mode : 0;
    if (groups) *groups = ctx ? ctx->shard_last_groups : 0;
}

int pa_cuda_nccl_wait(pa_cuda_ctx *ctx, void *comm, void *stream, uint32_t timeout_ms) {
    if (!ctx || !comm) return PA_CUDA_EINVAL;
    const NcclApi *api = nccl_api();
    if (!api) return fail(ctx, PA_CUDA_ENCCL, "libnccl.so.2 could not be opened");
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, PA_CUDA_ECUDA, "cudaSetDevice");
    return shard_wait(ctx, api, (ShardComm *) comm, pick(ctx, stream), timeout_ms);
}

int pa_cuda_shard_attn_allgather_merge(pa_cuda_plan *p, const uint16_t *Qs, void *comm, float *O, float *m, float *l,
                                       void *stream) {
    if (!p) return PA_CUDA_EINVAL;
    pa_cuda_ctx *ctx = p->ctx;
    auto *sc = (ShardComm *) comm;
    if (!sc || !O || !m || !l || (p->n_jobs && !Qs)) return fail(ctx, PA_CUDA_EINVAL, "null argument");
    if (sc->dead) return fail(ctx, PA_CUDA_ENCCL, "the communicator was aborted after a failed or overdue exchange");
    const NcclApi *api = nccl_api();
    if (!api) return fail(ctx, PA_CUDA_ENCCL, "libnccl.so.2 could not be opened");
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, PA_CUDA_ECUDA, "cudaSetDevice");
    const int world = sc->world;
    const uint32_t hd = p->sh.hd, ns = p->n_sets;
    const uint64_t rps = (uint64_t) p->sh.nkv * p->sh.rows;            // rows per output set
    const uint64_t rows = (uint64_t) ns * rps, part = rows * (hd + 2);   // floats of one rank's packed partial
    // exchange: the peer stores (small partials: no collective launch on the call's path), the all-gather moves N-1
    // partials into every rank, the two all-reduces ~2(N-1)/N of one
    const bool big = part * sizeof(float) >= kShardReduceBytes;
    int mode = ctx->shard_exchange ? ctx->shard_exchange : big ? (world > 2 ? 2 : 1) : 3;
    cudaStream_t st0 = pick(ctx, stream);
    if (mode == 3) {
        p2p_setup(ctx, api, sc, part, (rows + 7) / 8, st0);   // collective the first time (and when more room is needed)
        if (sc->dead) return fail(ctx, PA_CUDA_ENCCL, "the communicator was aborted while setting up the peer stores");
        if (sc->p2p_state != 1) mode = (big && world > 2) ? 2 : 1;
    }
    ctx->shard_last_mode = mode;
    if (mode == 3) {
        // the attention kernel, then one exchange kernel: its blocks merge this rank's rows, store them into every
        // rank's receive area (the half of this call's parity) and publish them, then fold every rank's rows
        const unsigned long long epoch = ++sc->p2p_calls;
        int rc = run_attention_sets(p, Qs, st0, 0, ns);
        if (rc) return rc;
        pa::mrg::XParams x{};
        x.Op = p->d_op;
        x.Mp = p->d_mp;
        x.Lp = p->d_lp;
        x.c_range = p->d_crange;
        x.op_stride = (uint64_t) p->sh.nkv * p->sh.rows * hd;
        x.ml_stride = (uint64_t) p->sh.nkv * p->sh.rows;
        x.rows_per_set = rps;
        x.n_sets = ns;
        x.push = sc->d_push;
        x.push_off = (epoch & 1) * (uint64_t) world * sc->p2p_cap;
        x.push_flag = sc->d_pflag;
        x.recv = (const float *) (sc->p2p_buf + sc->p2p_head) + (epoch & 1) * (uint64_t) world * sc->p2p_cap;
        x.flags = (const unsigned long long *) sc->p2p_buf;
        x.cap = sc->p2p_cap;
        x.blocks_cap = sc->p2p_blocks;
        x.epoch = epoch;
        x.world = (uint32_t) world;
        x.O = O;
        x.M = m;
        x.L = l;
        x.status = ctx->d_status;
        x.timeout_ns = ctx->timeout_ns;
        const unsigned blocks = (unsigned) ((rows + 7) / 8);
        if (blocks) {
            if (hd == 128) pa::mrg::shard_exchange_kernel<128><<<blocks, 256, 0, st0>>>(x);
            else pa::mrg::shard_exchange_kernel<256><<<blocks, 256, 0, st0>>>(x);
            PA_CK(cudaGetLastError(), "exchange kernel launch");
            ctx->launches++;
        }
        ctx->shard_last_groups = 1;
        if (ctx->shard_timeout_ms) {
            if ((rc = shard_wait(ctx, api, sc, st0, ctx->shard_timeout_ms))) return rc;
            return pa_cuda_status(ctx, st0);
        }
        return PA_CUDA_OK;
    }
    // set groups: each group's exchange overlaps the next group's kernels
    uint32_t G = ctx->shard_groups ? (uint32_t) ctx->shard_groups
               : (part * sizeof(float) >= kShardGroupBytes ? kShardGroups : 1u);
    G = std::max(1u, std::min(G, std::max(1u, ns)));
    ctx->shard_last_groups = (int) G;
    int rc = ensure_dev(ctx, ctx->d_shard, ctx->d_shard_bytes, part * sizeof(float));
    if (!rc && mode == 1) rc = ensure_dev(ctx, ctx->d_gathered, ctx->d_gathered_bytes, (size_t) world * part * sizeof(float));
    if (rc) return rc;
    cudaStream_t st = pick(ctx, stream), xs = st;
    if (G > 1) {
        if (!ctx->xstream) {
            // the highest priority: the block scheduler hands freed SMs to the exchange's kernels (NCCL, the fold)
            // before the remaining CTAs of the next group's attention kernel, so the exchange really overlaps it
            int least = 0, greatest = 0;
            PA_CK(cudaDeviceGetStreamPriorityRange(&least, &greatest), "stream priorities");
            PA_CK(cudaStreamCreateWithPriority(&ctx->xstream, cudaStreamNonBlocking, greatest), "exchange stream");
        }
        while (ctx->xev.size() < G + 1) {
            cudaEvent_t e;
            PA_CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event create");
            ctx->xev.push_back(e);
        }
        xs = ctx->xstream;
    }
    for (uint32_t g = 0; g < G; g++) {
        const uint32_t s0 = (uint32_t) ((uint64_t) ns * g / G), s1 = (uint32_t) ((uint64_t) ns * (g + 1) / G);
        if (s1 == s0) continue;
        const uint64_t r0 = (uint64_t) s0 * rps, rg = (uint64_t) (s1 - s0) * rps;
        // this rank's partial of the group's sets, packed O [rg][hd], m [rg], l [rg] (the layout the fold reads)
        float *pk = ctx->d_shard + r0 * (hd + 2), *pm = pk + rg * hd, *pl = pm + rg;
        if ((rc = run_plan_sets(p, Qs, pk, pm, pl, st, s0, s1))) return rc;
        if (G > 1) {
            PA_CK(cudaEventRecord(ctx->xev[g], st), "event record");
            PA_CK(cudaStreamWaitEvent(xs, ctx->xev[g], 0), "stream wait");
        }
        ncclResult_t r;
        if (mode == 1) {
            float *ga = ctx->d_gathered + (uint64_t) world * r0 * (hd + 2);
            if ((r = api->all_gather(pk, ga, rg * (hd + 2), ncclFloat32, sc->nc, xs)) != ncclSuccess)
                return nccl_fail(ctx, api, r, "ncclAllGather");
            if ((rc = pa_cuda_merge_gathered(ctx, hd, rg, (uint32_t) world, ga, O + r0 * hd, m + r0, l + r0, 0, xs))) return rc;
        } else {
            // the rows' maxima over all ranks straight into m, this rank's (O, l) moved to them, then summed into O, l
            if ((r = api->all_reduce(pm, m + r0, rg, ncclFloat32, ncclMax, sc->nc, xs)) != ncclSuccess)
                return nccl_fail(ctx, api, r, "ncclAllReduce (max)");
            const unsigned blocks = (unsigned) ((rg + 7) / 8);
            if (hd == 128) pa::mrg::rescale_to_kernel<128><<<blocks, 256, 0, xs>>>(pk, pm, pl, m + r0, rg);
            else pa::mrg::rescale_to_kernel<256><<<blocks, 256, 0, xs>>>(pk, pm, pl, m + r0, rg);
            PA_CK(cudaGetLastError(), "rescale launch");
            ctx->launches++;
            if ((r = api->group_start()) != ncclSuccess) return nccl_fail(ctx, api, r, "ncclGroupStart");
            ncclResult_t r1 = api->all_reduce(pk, O + r0 * hd, rg * hd, ncclFloat32, ncclSum, sc->nc, xs);
            ncclResult_t r2 = api->all_reduce(pl, l + r0, rg, ncclFloat32, ncclSum, sc->nc, xs);
            if ((r = api->group_end()) != ncclSuccess) return nccl_fail(ctx, api, r, "ncclGroupEnd");
            if (r1 != ncclSuccess || r2 != ncclSuccess) return nccl_fail(ctx, api, r1 != ncclSuccess ? r1 : r2, "ncclAllReduce (sum)");
        }
    }
    if (G > 1) {
        PA_CK(cudaEventRecord(ctx->xev[G], xs), "event record");
        PA_CK(cudaStreamWaitEvent(st, ctx->xev[G], 0), "stream wait");
    }
    if (ctx->shard_timeout_ms) return shard_wait(ctx, api, sc, st, ctx->shard_timeout_ms);
    return PA_CUDA_OK;
}

int pa_cuda_normalize(pa_cuda_ctx *ctx, uint32_t hd, uint64_t rows, const float *O, const float *m, const float *l,
                      uint16_t *Oh, float *lse, void *stream) {
    if (!ctx) return PA_CUDA_EINVAL;
    if (hd != 128 && hd != 256) return fail(ctx, PA_CUDA_EUNSUPPORTED, "hd must be 128 or 256");
    if (rows == 0) return PA_CUDA_OK;
    if (!O || !m || !l || !Oh || !lse) return fail(ctx, PA_CUDA_EINVAL, "null argument");
    cudaSetDevice(ctx->device);
    const unsigned blocks = (unsigned) ((rows + 7) / 8);
    if (hd == 128) pa::mrg::normalize_kernel<128><<<blocks, 256, 0, pick(ctx, stream)>>>(O, m, l, rows, Oh, lse);
    else pa::mrg::normalize_kernel<256><<<blocks, 256, 0, pick(ctx, stream)>>>(O, m, l, rows, Oh, lse);
    PA_CK(cudaGetLastError(), "normalize launch");
    ctx->launches++;
    return PA_CUDA_OK;
}

int pa_cuda_fold_reply(pa_cuda_ctx *ctx, uint32_t hd, uint64_t rows, const uint16_t *Oh, const float *lse, float *O,
                       float *m, float *l, void *stream) {
    if (!ctx) return PA_CUDA_EINVAL;
    if (hd != 128 && hd != 256) return fail(ctx, PA_CUDA_EUNSUPPORTED, "hd must be 128 or 256");
    if (rows == 0) return PA_CUDA_OK;
    if (!Oh || !lse || !O || !m || !l) return fail(ctx, PA_CUDA_EINVAL, "null argument");
    cudaSetDevice(ctx->device);
    const unsigned blocks = (unsigned) ((rows + 7) / 8);
    if (hd == 128) pa::mrg::fold_reply_kernel<128><<<blocks, 256, 0, pick(ctx, stream)>>>(Oh, lse, rows, O, m, l);
    else pa::mrg::fold_reply_kernel<256><<<blocks, 256, 0, pick(ctx, stream)>>>(Oh, lse, rows, O, m, l);
    PA_CK(cudaGetLastError(), "fold_reply launch");
    ctx->launches++;
    return PA_CUDA_OK;
}

// ------------------------------------------------------------------------------------------ pa::engine
int pa_cuda_alloc_page(pa_cuda_ctx *ctx, size_t bytes, pa_cuda_page *pg) {
    if (!ctx || !pg) return PA_CUDA_EINVAL;
    cudaSetDevice(ctx->device);
    uint8_t *k = nullptr, *v = nullptr;
    const size_t n = (bytes + 4095) / 4096 * 4096 + 64;   // +64: readable slack past the last row
    cudaError_t e = cudaMallocManaged((void **) &k, n, cudaMemAttachGlobal);
    if (e == cudaSuccess) e = cudaMallocManaged((void **) &v, n, cudaMemAttachGlobal);
    if (e != cudaSuccess) {
        if (k) cudaFree(k);
        return fail(ctx, PA_CUDA_ENOMEM, std::string("page allocation: ") + cudaGetErrorString(e));
    }
#if CUDART_VERSION >= 13000
    cudaMemLocation loc{cudaMemLocationTypeDevice, ctx->device};
    cudaMemAdvise(k, n, cudaMemAdviseSetPreferredLocation, loc);
    cudaMemAdvise(v, n, cudaMemAdviseSetPreferredLocation, loc);
#else
    cudaMemAdvise(k, n, cudaMemAdviseSetPreferredLocation, ctx->device);
    cudaMemAdvise(v, n, cudaMemAdviseSetPreferredLocation, ctx->device);
#endif
    cudaGetLastError();
    pg->k = k;
    pg->v = v;
    pg->hk = k;
    pg->hv = v;
    return PA_CUDA_OK;
}

void pa_cuda_free_page(pa_cuda_ctx *ctx, pa_cuda_page *pg) {
    if (!ctx || !pg) return;
    cudaSetDevice(ctx->device);
    if (ctx->eng_active) cudaStreamSynchronize(ctx->stream);
    ctx->eng_resident.erase((uintptr_t) pg->k);
    if (pg->k) cudaFree(pg->k);
    if (pg->v) cudaFree(pg->v);
    pg->k = pg->v = nullptr;
    pg->hk = pg->hv = nullptr;
}

}  // extern "C"

namespace {

// One engine call's plan from the cache (created on a miss, the least recently used one evicted past kEngCache), with
// the staging buffers sized for it. Cached graphs capture the staging buffers' addresses: a reallocation drops them.
int eng_prepare(pa_cuda_ctx *ctx, const pa_cuda_page *pages, const uint32_t *nkeys, int n_pages, const pa_cuda_shape *shape,
                int ng, int ntok, pa_cuda_shape &sh, int &nt, EngEntry *&entry) {
    if (ng < 1 || n_pages < 0 || (n_pages && (!pages || !nkeys)) || !shape)
        return fail(ctx, PA_CUDA_EINVAL, "bad begin arguments");
    cudaSetDevice(ctx->device);
    const int NR = 48;
    sh = *shape;
    nt = (ng == 1 && ntok >= 1 && ntok < 8) ? ntok : 0;   // packed real rows (pa-metal.mm:627-646)
    sh.rows = nt ? 6u * (uint32_t) nt : (uint32_t) NR;
    int rc = check_shape(ctx, &sh);
    if (rc) return rc;
    // the context's kernel choice and QK arithmetic are part of the key: a call after pa_cuda_set_kernel or
    // pa_cuda_set_qk_domain gets a plan built under the new setting, not a cached one
    std::vector<uint64_t> key = {sh.hd, sh.nkv, sh.rows, sh.quant, sh.rs, sh.hb, (uint64_t) ng, (uint64_t) nt,
                                 (uint64_t) (uint32_t) ctx->kernel_choice, (uint64_t) (uint32_t) ctx->qk_domain,
                                 (uint64_t) n_pages};
    for (int i = 0; i < n_pages; i++) {
        key.push_back((uint64_t) (uintptr_t) pages[i].k);
        key.push_back((uint64_t) (uintptr_t) pages[i].v);
        key.push_back(nkeys[i]);
    }
    entry = nullptr;
    for (auto &e : ctx->eng_cache)
        if (e.key == key) { entry = &e; break; }
    if (!entry) {
        // evict least recently used entries while the cache is full (by count or by plan scratch)
        auto held = [&]() {
            size_t b = 0;
            for (auto &e : ctx->eng_cache) b += e.plan ? e.plan->scratch : 0;
            return b;
        };
        while (!ctx->eng_cache.empty() && (ctx->eng_cache.size() >= kEngCache || held() > kEngCacheBytes)) {
            auto lru = std::min_element(ctx->eng_cache.begin(), ctx->eng_cache.end(),
                                        [](const EngEntry &a, const EngEntry &b) { return a.used < b.used; });
            cudaStreamSynchronize(ctx->stream);
            if (lru->graph) cudaGraphExecDestroy(lru->graph);
            if (lru->plan) pa_cuda_plan_destroy(lru->plan);
            ctx->eng_cache.erase(lru);
        }
        std::vector<pa_cuda_seg> segs;
        for (int g = 0; g < ng; g++)
            for (int i = 0; i < n_pages; i++)
                if (nkeys[i]) segs.push_back(pa_cuda_seg{pages[i].k, pages[i].v, nkeys[i], (uint32_t) g});
        pa_cuda_plan *plan = nullptr;
        if ((rc = pa_cuda_plan_create(ctx, &sh, (uint32_t) ng, segs.data(), (uint32_t) segs.size(), 0, &plan))) return rc;
        ctx->eng_cache.push_back(EngEntry{});
        entry = &ctx->eng_cache.back();
        entry->key = std::move(key);
        entry->plan = plan;
    }
    entry->used = ++ctx->eng_tick;
    const size_t rows = (size_t) ng * sh.nkv * sh.rows;
    const size_t qb = rows * sh.hd * 2, ob = rows * sh.hd * 4, mb = rows * 4;
    const void *before[4] = {ctx->h_q, ctx->h_out, ctx->d_q, ctx->d_out};
    if ((rc = ensure_host(ctx, ctx->h_q, ctx->h_q_bytes, qb))) return rc;
    if ((rc = ensure_host(ctx, ctx->h_out, ctx->h_out_bytes, ob + 2 * mb + 16))) return rc;
    if ((rc = ensure_dev(ctx, ctx->d_q, ctx->d_q_bytes, qb))) return rc;
    if ((rc = ensure_dev(ctx, ctx->d_out, ctx->d_out_bytes, ob + 2 * mb))) return rc;
    if (before[0] != ctx->h_q || before[1] != ctx->h_out || before[2] != ctx->d_q || before[3] != ctx->d_out)
        for (auto &e : ctx->eng_cache)
            if (e.graph) { cudaGraphExecDestroy(e.graph); e.graph = nullptr; }
    return PA_CUDA_OK;
}

// Stream-ordered migration of the rows the host wrote into managed pages since the last call. The host writes pages only
// by APPEND (rows past the keys already held) or after a TRUNCATE (the page shrinks, then grows again), so a page whose
// key count is what was prefetched last is skipped: a steady decode step issues no prefetch at all. The prefetch is only
// a hint: rows the host rewrote without changing the count (TRUNCATE, then APPEND of as many rows) still reach the GPU
// correctly through managed memory's on-demand migration.
void eng_prefetch(pa_cuda_ctx *ctx, const pa_cuda_page *pages, const uint32_t *nkeys, int n_pages, uint64_t rs) {
    for (int i = 0; i < n_pages; i++) {
        auto it = ctx->eng_resident.find((uintptr_t) pages[i].k);
        const uint32_t had = it == ctx->eng_resident.end() ? 0u : it->second, now = nkeys[i];
        if (it != ctx->eng_resident.end() && had == now) continue;
        const size_t lo = now > had ? (size_t) had * rs : 0, hi = (size_t) now * rs;
        ctx->eng_resident[(uintptr_t) pages[i].k] = now;
        if (hi <= lo) continue;
#if CUDART_VERSION >= 13000
        cudaMemLocation loc{cudaMemLocationTypeDevice, ctx->device};
        cudaMemPrefetchAsync(pages[i].k + lo, hi - lo, loc, 0, ctx->stream);
        cudaMemPrefetchAsync(pages[i].v + lo, hi - lo, loc, 0, ctx->stream);
#else
        cudaMemPrefetchAsync(pages[i].k + lo, hi - lo, ctx->device, ctx->stream);
        cudaMemPrefetchAsync(pages[i].v + lo, hi - lo, ctx->device, ctx->stream);
#endif
    }
    cudaGetLastError();
}

// the device part of one engine call: Q up, the plan's kernels, (O, m, l) back
int eng_enqueue(pa_cuda_ctx *ctx, pa_cuda_plan *plan, const pa_cuda_shape &sh, int ng) {
    const size_t rows = (size_t) ng * sh.nkv * sh.rows;
    const size_t qb = rows * sh.hd * 2, ob = rows * sh.hd * 4, mb = rows * 4;
    PA_CK(cudaMemcpyAsync(ctx->d_q, ctx->h_q, qb, cudaMemcpyHostToDevice, ctx->stream), "Q to device");
    float *dO = ctx->d_out, *dm = (float *) ((char *) ctx->d_out + ob), *dl = dm + rows;
    int rc = run_plan(plan, ctx->d_q, dO, dm, dl, ctx->stream);
    if (rc) return rc;
    PA_CK(cudaMemcpyAsync(ctx->h_out, ctx->d_out, ob + 2 * mb, cudaMemcpyDeviceToHost, ctx->stream), "O to host");
    // the status word rides with the readback, so end() needs no second synchronising copy
    PA_CK(cudaMemcpyAsync((char *) ctx->h_out + ob + 2 * mb, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream),
          "status to host");
    return PA_CUDA_OK;
}

}  // namespace

extern "C" {

int pa_cuda_begin(pa_cuda_ctx *ctx, const pa_cuda_page *pages, const uint32_t *nkeys, int n_pages,
                  const uint16_t *Qs_host, const pa_cuda_shape *shape, int ng, int ntok) {
    if (!ctx) return PA_CUDA_EINVAL;
    if (ctx->eng_active) return fail(ctx, PA_CUDA_EINVAL, "begin while a call is in flight (call end first)");
    if (!Qs_host) return fail(ctx, PA_CUDA_EINVAL, "bad begin arguments");
    const auto t_call = std::chrono::steady_clock::now();   // end() reports the time from here (plan lookup, Q packing)
    pa_cuda_shape sh;
    int nt = 0;
    EngEntry *entry = nullptr;
    int rc = eng_prepare(ctx, pages, nkeys, n_pages, shape, ng, ntok, sh, nt, entry);
    if (rc) return rc;
    ctx->eng_plan = entry->plan;
    const int NR = 48;
    const uint32_t nkv = sh.nkv, hd = sh.hd;
    // pack Q: wire row r = g*8 + t of head h; packed (nt) row = g*nt + t
    for (int gi = 0; gi < ng; gi++)
        for (uint32_t h = 0; h < nkv; h++) {
            const uint16_t *src = Qs_host + ((size_t) gi * nkv + h) * NR * hd;
            uint16_t *dst = ctx->h_q + ((size_t) gi * nkv + h) * sh.rows * hd;
            if (!nt) memcpy(dst, src, (size_t) NR * hd * 2);
            else
                for (int gg = 0; gg < 6; gg++) memcpy(dst + (size_t) gg * nt * hd, src + (size_t) gg * 8 * hd, (size_t) nt * hd * 2);
        }
    eng_prefetch(ctx, pages, nkeys, n_pages, sh.rs);
    ctx->t_begin = t_call;
    PA_CK(cudaEventRecord(ctx->ev_begin, ctx->stream), "event");
    if (entry->graph && !entry->plan->profile) {   // armed: one graph launch replays the whole call
        PA_CK(cudaGraphLaunch(entry->graph, ctx->stream), "graph launch");
        ctx->launches += entry->graph_launches;
        ctx->eng_graph_calls++;
    } else if ((rc = eng_enqueue(ctx, entry->plan, sh, ng))) {
        return rc;
    }
    PA_CK(cudaEventRecord(ctx->ev_end, ctx->stream), "event");
    ctx->eng_ng = ng;
    ctx->eng_nt = nt;
    ctx->eng_rows = (int) sh.rows;
    ctx->eng_nkv = (int) nkv;
    ctx->eng_hd = (int) hd;
    ctx->eng_active = true;
    return PA_CUDA_OK;
}

int pa_cuda_arm(pa_cuda_ctx *ctx, const pa_cuda_page *pages, const uint32_t *nkeys, int n_pages,
                const pa_cuda_shape *shape, int ntok) {
    if (!ctx) return PA_CUDA_EINVAL;
    if (ctx->eng_active) return fail(ctx, PA_CUDA_EINVAL, "arm while a call is in flight (call end first)");
    pa_cuda_shape sh;
    int nt = 0;
    EngEntry *entry = nullptr;
    int rc = eng_prepare(ctx, pages, nkeys, n_pages, shape, 1, ntok, sh, nt, entry);
    if (rc) return rc;
    eng_prefetch(ctx, pages, nkeys, n_pages, sh.rs);
    if (entry->graph) return PA_CUDA_OK;
    // capture the call on the context's stream (nothing of this thread is in flight on it between end and begin)
    const uint64_t launches0 = ctx->launches;
    cudaGraph_t g = nullptr;
    PA_CK(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    rc = eng_enqueue(ctx, entry->plan, sh, 1);
    const cudaError_t ec = cudaStreamEndCapture(ctx->stream, &g);
    const uint64_t per_run = ctx->launches - launches0;
    ctx->launches = launches0;   // captured, not run
    if (rc || ec != cudaSuccess || !g) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return rc ? rc : cuda_fail(ctx, ec, "capture of the armed call");
    }
    cudaGraphExec_t ex = nullptr;
    const cudaError_t ei = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(ctx, ei, "instantiating the armed call");
    }
    entry->graph = ex;
    entry->graph_launches = per_run;
    return PA_CUDA_OK;
}

uint64_t pa_cuda_graph_calls(const pa_cuda_ctx *ctx) { return ctx ? ctx->eng_graph_calls : 0; }

double pa_cuda_end(pa_cuda_ctx *ctx, float *O, float *m, float *l) {
    if (!ctx || !ctx->eng_active) return -1;
    ctx->eng_active = false;
    const int NR = 48, ng = ctx->eng_ng, nt = ctx->eng_nt, nkv = ctx->eng_nkv, hd = ctx->eng_hd, rows = ctx->eng_rows;
    const size_t out_rows = (size_t) ng * nkv * NR;
    cudaError_t e = cudaEventSynchronize(ctx->ev_end);
    const size_t prow = (size_t) ng * nkv * rows;
    int st = PA_CUDA_ECUDA;
    if (e == cudaSuccess) {
        const int h = *reinterpret_cast<const volatile int *>((const char *) ctx->h_out + prow * hd * 4 + 2 * prow * 4);
        st = PA_CUDA_OK;
        if (h != pa::ST_OK) {   // a kernel of this call gave up a bounded wait: clear the word for the next call
            cudaMemsetAsync(ctx->d_status, 0, sizeof(int), ctx->stream);
            cudaStreamSynchronize(ctx->stream);
            st = fail(ctx, PA_CUDA_ETIMEOUT, "a kernel gave up a bounded wait (code " + std::to_string(h) + ")");
        }
    }
    if (e != cudaSuccess || st != PA_CUDA_OK) {
        for (size_t r = 0; r < out_rows; r++) { m[r] = -INFINITY; l[r] = 0; }
        if (e != cudaSuccess) ctx->err = std::string("GPU call failed: ") + cudaGetErrorString(e);
        return -1;
    }
    float ms = 0;
    cudaEventElapsedTime(&ms, ctx->ev_begin, ctx->ev_end);
    ctx->last_exec_ms = ms;
    const float *hO = ctx->h_out, *hm = hO + prow * hd, *hl = hm + prow;
    for (int gi = 0; gi < ng; gi++)
        for (int h = 0; h < nkv; h++)
            for (int r = 0; r < NR; r++) {
                const size_t orow = ((size_t) gi * nkv + h) * NR + r;
                int pr = r;
                if (nt) pr = (r % 8) < nt ? (r / 8) * nt + (r % 8) : -1;
                if (pr < 0) {
                    memset(O + orow * hd, 0, (size_t) hd * 4);
                    m[orow] = -INFINITY;
                    l[orow] = 0;
                    continue;
                }
                const size_t srow = ((size_t) gi * nkv + h) * rows + pr;
                memcpy(O + orow * hd, hO + srow * hd, (size_t) hd * 4);
                m[orow] = hm[srow];
                l[orow] = hl[srow];
            }
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - ctx->t_begin).count();
}

double pa_cuda_exec_ms(const pa_cuda_ctx *ctx) { return ctx ? ctx->last_exec_ms : 0; }

}  // extern "C"

// ====================================================================================================== no allocation
// pa_cuda_attn_noalloc: the split-K kernel with its scratch (the chunk partials, the job list, the status word) in a
// fixed device array, for callers that cannot allocate device memory (see include/pa_cuda.h).
namespace {

constexpr size_t kNaBytes = 16u << 20;   // per GPU; held by every GPU that loads the library until the process exits
constexpr uint32_t kNaMaxJobs = 2048;
constexpr size_t kNaStatus = 0;          // int: bounded-wait status of the call
constexpr size_t kNaRange = 256;         // uint32_t[2]: the merge's part range [0, n_jobs)
constexpr size_t kNaJobs = 512;          // pa::dec::Job[kNaMaxJobs]
constexpr size_t kNaParts = (kNaJobs + kNaMaxJobs * sizeof(pa::dec::Job) + 255) / 256 * 256;   // partials

static __device__ __align__(256) uint8_t g_na_scratch[kNaBytes];

// the device address of g_na_scratch per device (set up by the first call on that device; a host-side name of a
// __device__ array is not a device address). The address belongs to the device's primary context: after
// cudaDeviceReset it would be stale, so a process that resets a device does not use this entry point afterwards.
std::mutex g_na_mu;
uint8_t *g_na_ptr[128] = {};

// writes this call's job list, part range and a zero status into the scratch (the array keeps the previous call's
// contents otherwise)
__global__ void noalloc_setup_kernel(uint8_t *base, const uint8_t *K, const uint8_t *V, uint32_t nk, uint32_t chunk,
                                     uint32_t n_jobs) {
    pa::dec::Job *jobs = reinterpret_cast<pa::dec::Job *>(base + kNaJobs);
    for (uint32_t i = threadIdx.x; i < n_jobs; i += blockDim.x) {
        pa::dec::Job j;
        j.k = K;
        j.v = V;
        j.key0 = i * chunk;
        j.nk = min(chunk, nk - i * chunk);
        j.set = 0;
        j.slot = i;
        j.seg = 0;
        j.pad_ = 0;
        jobs[i] = j;
    }
    if (threadIdx.x == 0) {
        *reinterpret_cast<int *>(base + kNaStatus) = pa::ST_OK;
        uint32_t *range = reinterpret_cast<uint32_t *>(base + kNaRange);
        range[0] = 0;
        range[1] = n_jobs;
    }
}

int na_fail(const char **why, int code, const char *msg) {
    if (why) *why = msg;
    return code;
}

}  // namespace

extern "C" int pa_cuda_attn_noalloc(const pa_cuda_shape *shape, const uint16_t *Qs, const uint8_t *K, const uint8_t *V,
                                    uint32_t nk, float *O, float *m, float *l, void *stream, const char **why) {
    if (why) *why = "";
    if (!shape || !O || !m || !l || (nk && (!Qs || !K || !V))) return na_fail(why, PA_CUDA_EINVAL, "null argument");
    if (check_shape(nullptr, shape) != PA_CUDA_OK)
        return na_fail(why, PA_CUDA_EUNSUPPORTED, "shape: hd 128/256, F16, Q8_0 or Q4_0 rows, hb of the format, rs >= nkv*hb "
                                                  "and a multiple of 16");
    if (nk && (((uintptr_t) K | (uintptr_t) V) & 15)) return na_fail(why, PA_CUDA_EINVAL, "K/V not 16-byte aligned");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return na_fail(why, PA_CUDA_ECUDA, "cudaGetDevice");
    uint8_t *base;
    {
        std::lock_guard<std::mutex> lk(g_na_mu);
        if (!g_na_ptr[dev]) {
            void *ptr = nullptr;
            if (cudaGetSymbolAddress(&ptr, g_na_scratch) != cudaSuccess || !ptr)
                return na_fail(why, PA_CUDA_ECUDA, "cudaGetSymbolAddress of the fixed scratch failed");
            g_na_ptr[dev] = (uint8_t *) ptr;
        }
        base = g_na_ptr[dev];
    }
    const uint64_t rows_all = (uint64_t) shape->nkv * shape->rows;
    const uint64_t slot_bytes = rows_all * (shape->hd + 2) * 4;
    const uint64_t max_slots = std::min<uint64_t>(kNaMaxJobs, (kNaBytes - kNaParts) / slot_bytes);
    if (max_slots == 0)
        return na_fail(why, PA_CUDA_EUNSUPPORTED,
                       "nkv * rows * (hd + 2) * 4 bytes (one chunk partial) exceed the 16 MiB fixed scratch");
    pa_cuda_plan p;   // launch shape only: no allocation
    p.ctx = nullptr;
    p.sh = *shape;
    p.n_sets = 1;
    if (plan_decode_shape(nullptr, &p) != PA_CUDA_OK)
        return na_fail(why, PA_CUDA_EUNSUPPORTED, "no head grouping of this shape fits the split-K kernel");
    int n_sm = 148;
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    uint32_t chunk = 0, n_jobs = 0;
    if (nk) {
        const uint64_t per_y = std::max<uint64_t>(1, (uint64_t) n_sm * 16 / std::max<uint32_t>(1, p.grid_y));
        chunk = (uint32_t) std::min<uint64_t>(16384, std::max<uint64_t>(128, (nk + per_y - 1) / per_y));
        chunk = (chunk + 63) / 64 * 64;
        if ((nk + chunk - 1) / chunk > max_slots) chunk = (uint32_t) (((nk + max_slots - 1) / max_slots + 63) / 64 * 64);
        n_jobs = (nk + chunk - 1) / chunk;
    }
    p.n_jobs = p.n_slots = n_jobs;
    cudaStream_t st = (cudaStream_t) stream;
    noalloc_setup_kernel<<<1, 256, 0, st>>>(base, K, V, nk, chunk, n_jobs);
    if (cudaGetLastError() != cudaSuccess) return na_fail(why, PA_CUDA_ECUDA, "setup kernel launch failed");
    float *Op = reinterpret_cast<float *>(base + kNaParts);
    float *Mp = Op + (uint64_t) n_jobs * rows_all * shape->hd, *Lp = Mp + (uint64_t) n_jobs * rows_all;
    int *status = reinterpret_cast<int *>(base + kNaStatus);
    if (n_jobs) {
        pa::dec::Params prm{};
        prm.jobs = reinterpret_cast<const pa::dec::Job *>(base + kNaJobs);
        prm.Qs = Qs;
        prm.Op = Op;
        prm.Mp = Mp;
        prm.Lp = Lp;
        prm.status = status;
        prm.rs = shape->rs;
        prm.hb = shape->hb;
        prm.nkv = shape->nkv;
        prm.rows = shape->rows;
        prm.hg = p.hg;
        prm.rgc = p.rgc;
        prm.n_rg = p.n_rg;
        prm.row = p.row;
        prm.gs = p.gs;
        prm.n_jobs = n_jobs;
        prm.n_consumers = p.n_consumers;
        prm.timeout_ns = 2000000000ull;
        prm.stall = 0;
        cudaError_t e;
        e = launch_decode_any(&p, n_jobs, prm, st, shape->hd, shape->quant);
        if (e != cudaSuccess) return na_fail(why, PA_CUDA_ECUDA, "split-K kernel launch failed");
    }
    pa::mrg::Params mp{};
    mp.Op = Op;
    mp.Mp = Mp;
    mp.Lp = Lp;
    mp.c_range = reinterpret_cast<const uint32_t *>(base + kNaRange);
    mp.n_parts = n_jobs;
    mp.op_stride = rows_all * shape->hd;
    mp.ml_stride = rows_all;
    mp.set_rows = 0;
    mp.O = O;
    mp.M = m;
    mp.L = l;
    mp.rows_per_set = rows_all;
    mp.n_sets = 1;
    mp.fold = 0;
    if ((shape->hd == 128 ? launch_merge<128>(mp, st, n_sm) : launch_merge<256>(mp, st, n_sm)) != cudaSuccess)
        return na_fail(why, PA_CUDA_ECUDA, "merge kernel launch failed");
    if (cudaStreamSynchronize(st) != cudaSuccess) return na_fail(why, PA_CUDA_ECUDA, "stream synchronize failed");
    int h = 0;
    if (cudaMemcpy(&h, status, sizeof h, cudaMemcpyDeviceToHost) != cudaSuccess)
        return na_fail(why, PA_CUDA_ECUDA, "status read failed");
    if (h != pa::ST_OK) return na_fail(why, PA_CUDA_ETIMEOUT, "a kernel gave up a bounded wait");
    return PA_CUDA_OK;
}
