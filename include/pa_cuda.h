/* pa_cuda.h - C ABI of libpacuda.so, the B200 (sm_100a) engine for Backburner's phone-attn hot path: partial attention
 * over an offloaded, position-contiguous segment of a Q8_0 / Q4_0 KV cache, returning the unnormalised partial
 * (O, m, l) that the host merges with its own by log-sum-exp.
 *
 * Every entry point is plain C: device or host pointers and sizes, no framework types. Reference interfaces each one
 * replaces (paths inside the reference repository):
 *   pa_cuda_available      sme2_available                 phone-attn/phone-attn.h:67
 *   pa_cuda_attn_partial   sme_attn_partial               phone-attn/phone-attn.h:65-66, scripts/sme/sme_attn.c:271-306
 *   pa_cuda_attn, plans    sme_attn_pipe (all heads)      phone-attn/phone-attn.h:69-70, scripts/sme/sme_attn.c:448-463
 *                          + the engine's page batching   phone-attn/pa-metal.mm:627-714
 *   pa_cuda_merge          pa_merge / pa_merge_big        phone-attn/pa-metal.mm:137-159, 490-524
 *                          merge_partial                  phone-attn/phone-attn.h:231-239
 *   pa_cuda_merge_gathered the multi-phone merge           docs/TWO-PHONES.md:14-18 (host loop in the absent llama.cpp)
 *   pa_cuda_shard_attn_allgather_merge, pa_cuda_nccl_*
 *                          the same split with the exchange   docs/TWO-PHONES.md:14-18 (one NCCL all-gather per call)
 *   pa_cuda_normalize      attn_core's O/l, lse           phone-attn/phone-attn.h:651-655
 *   pa_cuda_fold_reply     co-attention slot of a reply   phone-attn/phone-attn.h:18-20 (host merge in the absent llama.cpp)
 *   pa_cuda_scale_q        f16(q * scale)                 phone-attn/phone-attn.h:595-599, scripts/sme/sme_attn.c:276-280
 *   pa_cuda_set_qk_domain  sme_qk_i8blk + i8_combine      scripts/sme/sme_attn.c:465-508 (int8-domain QK, opt-in)
 *   pa_cuda_alloc_page,
 *   pa_cuda_free_page,
 *   pa_cuda_begin,
 *   pa_cuda_end            pa::engine                     phone-attn/phone-attn.h:166-183 (pa-metal.mm:804-953)
 *   pa_cuda_arm            engine::arm (pre-armed call)   phone-attn/phone-attn.h:179-182, pa-metal.mm:716-765
 *
 * Data layout (the reference's, unchanged):
 *   K/V rows: key position j, KV head h at base + j*rs + h*hb; Q8_0 head = hd/32 blocks of (f16 d, 32 x int8),
 *   Q4_0 head = hd/32 blocks of (f16 d, 16 bytes: byte i = elem i | elem i+16 << 4, value (n - 8) * d).
 *   Qs: f16(q * scale) [set][nkv][rows][hd]; O: fp32 [set][nkv][rows][hd]; m, l: fp32 [set][nkv][rows].
 *   O is unnormalised: O = sum_j exp(s_j - m) v_j, l = sum_j exp(s_j - m), m = max_j s_j; no keys: m = -inf, l = 0.
 *
 * Errors: functions return PA_CUDA_OK (0) or a negative code; pa_cuda_last_error() gives the text. Kernels never trap:
 * a bounded wait that runs out records a code on the device, which pa_cuda_status() returns.
 * Threading: a context is used by one host thread at a time (as pa::server's session thread uses its engine).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PA_CUDA_ABI_VERSION 1

enum {
    PA_CUDA_OK = 0,
    PA_CUDA_EINVAL = -1,       /* bad argument (message says which) */
    PA_CUDA_ECUDA = -2,        /* a CUDA call failed */
    PA_CUDA_ENOMEM = -3,       /* device or host allocation failed */
    PA_CUDA_ETIMEOUT = -4,     /* a kernel's bounded wait ran out (the context stays usable) */
    PA_CUDA_EUNSUPPORTED = -5, /* shape the kernels do not cover */
    PA_CUDA_ENCCL = -6         /* an NCCL call failed */
};

/* config_req.is_q8 (phone-attn/phone-attn.h:15) */
enum { PA_CUDA_F16 = 0, PA_CUDA_Q8_0 = 1, PA_CUDA_Q4_0 = 2 };

typedef struct pa_cuda_ctx pa_cuda_ctx;
typedef struct pa_cuda_plan pa_cuda_plan;

/* Geometry of a call. hd: 128 or 256. nkv: KV heads (1..16). rows: query rows per KV head (tokens x GQA group).
 * quant: PA_CUDA_Q8_0 or PA_CUDA_Q4_0. rs: bytes per key position (multiple of 16). hb: bytes per head in a position
 * (hd/32*34 for Q8_0, hd/32*18 for Q4_0). K/V base pointers must be 16-byte aligned. */
typedef struct pa_cuda_shape {
    uint32_t hd, nkv, rows, quant;
    uint64_t rs, hb;
} pa_cuda_shape;

/* A run of nk consecutive key positions (a page, or one layer's shard) whose partial folds into output set `set`.
 * k, v: device pointers to the run's first position. */
typedef struct pa_cuda_seg {
    const uint8_t *k, *v;
    uint32_t nk, set;
} pa_cuda_seg;

/* pa::page (phone-attn/phone-attn.h:163): k, v are host-writable and device-readable (managed memory). */
typedef struct pa_cuda_page {
    uint8_t *k, *v;
    void *hk, *hv;
} pa_cuda_page;

/* 1 if a device of compute capability 10.x (B200, sm_100a) is visible and the kernels load on it. */
int pa_cuda_available(void);
int pa_cuda_abi_version(void);

int pa_cuda_create(int device, pa_cuda_ctx **out);
void pa_cuda_destroy(pa_cuda_ctx *ctx);
const char *pa_cuda_last_error(const pa_cuda_ctx *ctx);
/* Synchronise `stream` (a cudaStream_t; NULL = the context's stream), then return and clear the device status word:
 * PA_CUDA_OK, or PA_CUDA_ETIMEOUT if a kernel gave up a bounded wait since the last call. */
int pa_cuda_status(pa_cuda_ctx *ctx, void *stream);
/* Bound on every in-kernel wait (default 2 s). */
void pa_cuda_set_timeout_ns(pa_cuda_ctx *ctx, uint64_t ns);
/* Kernel selection for plans created afterwards (as the reference engine's PA_BIG_KERNEL / PA_BIG_MIN_NG switches,
 * phone-attn/pa-metal.mm:818-821): 0 = by shape (default, quantised rows: the tcgen05 kernels from 9 query rows per KV
 * head, on single CTAs up to 256 rows at hd 128 and 128 at hd 256, on CTA pairs above; the split-K mma.sync kernel
 * otherwise), 1 = always the split-K kernel, 2 = the tcgen05 kernel on single CTAs, 3 = the tcgen05 kernel on CTA
 * pairs (hd 128 or 256 for both). */
void pa_cuda_set_kernel(pa_cuda_ctx *ctx, int which);
/* QK arithmetic for plans created afterwards. PA_CUDA_QK_F16 (default): K dequantised to f16(d*q) and S = Qs.K^T in
 * f16 with fp32 accumulation (sme_attn_partial, scripts/sme/sme_attn.c:274-306). PA_CUDA_QK_INT8: the reference's
 * compressed-domain QK (sme_qk_i8blk + i8_combine, scripts/sme/sme_attn.c:465-508): Q quantised per 32-block by the
 * Q8_0 rule (d = f16(max|x|/127), q = rint(x/d)), per-block int32 dot products with the Q8_0 K bytes on the s8 tensor
 * path, S = sum_b T_b * dq_b * dk_b in fp32; softmax and P.V unchanged. Q8_0 rows only and on the split-K kernel at
 * every row count: creating a plan for other rows, or with pa_cuda_set_kernel 2 / 3, fails with PA_CUDA_EUNSUPPORTED.
 * Its scores differ from the f16 path's by Q's int8 rounding (about 1e-2 of O on the reference's distributions), so it
 * is opt-in. pa_cuda_attn_noalloc (no context) always uses PA_CUDA_QK_F16. */
#define PA_CUDA_QK_F16 0
#define PA_CUDA_QK_INT8 1
void pa_cuda_set_qk_domain(pa_cuda_ctx *ctx, int domain);
/* Failure-detection test hook: while on, the decode kernel's consumer warps (the tcgen05 kernels' softmax warps) first
 * wait on a barrier that nothing completes, so their bounded wait runs out after the timeout; the kernel records
 * PA_CUDA_ETIMEOUT, every role unwinds and returns without trapping, and the context stays usable. Off by default. */
void pa_cuda_set_stall_test(pa_cuda_ctx *ctx, int on);
/* Kernel launches made by this context since it was created (the bench reports launches per step from it). */
uint64_t pa_cuda_launch_count(const pa_cuda_ctx *ctx);

/* ---- plans: the split of a call into per-chunk jobs, built once and run many times (CUDA-graph capturable).
 * chunk_keys: keys per CTA job (0 = chosen from the device's SM count). The plan owns its scratch (the chunk
 * partials, pa_cuda_plan_scratch_bytes()) in device memory. */
int pa_cuda_plan_create(pa_cuda_ctx *ctx, const pa_cuda_shape *shape, uint32_t n_sets, const pa_cuda_seg *segs,
                        uint32_t n_segs, uint32_t chunk_keys, pa_cuda_plan **out);
size_t pa_cuda_plan_scratch_bytes(const pa_cuda_plan *plan);
uint32_t pa_cuda_plan_jobs(const pa_cuda_plan *plan);
/* kernel launches one pa_cuda_plan_run makes */
uint32_t pa_cuda_plan_launches(const pa_cuda_plan *plan);
/* name of the plan's attention-kernel instance, e.g. "pa::pre::prefill_pair_kernel<1,2>" (static storage) */
const char *pa_cuda_plan_kernel(const pa_cuda_plan *plan);
/* Qs, O, m, l: device pointers laid out [set][nkv][rows]...; stream: cudaStream_t (NULL = the context's stream).
 * Asynchronous. */
int pa_cuda_plan_run(pa_cuda_plan *plan, const uint16_t *Qs, float *O, float *m, float *l, void *stream);
void pa_cuda_plan_destroy(pa_cuda_plan *plan);
/* Kernel timing (as the reference engine reads GPUStartTime/GPUEndTime, phone-attn/pa-metal.mm:938-945): with
 * max_runs > 0, each of the next max_runs runs records CUDA events around its decode kernel on the run's stream;
 * pa_cuda_plan_kernel_ms waits for them, returns their summed duration and count, and rearms. 0 turns it off. */
int pa_cuda_plan_profile(pa_cuda_plan *plan, uint32_t max_runs);
int pa_cuda_plan_kernel_ms(pa_cuda_plan *plan, double *total_ms, uint32_t *n_runs);

/* One-shot: plan, run, free (allocates; synchronises the stream before freeing the plan). */
int pa_cuda_attn(pa_cuda_ctx *ctx, const pa_cuda_shape *shape, const uint16_t *Qs, uint32_t n_sets,
                 const pa_cuda_seg *segs, uint32_t n_segs, float *O, float *m, float *l, void *stream);

/* sme_attn_partial for all heads of one segment: Q fp32 [nkv][rows][hd] unscaled (device), scale applied as
 * f16(q * scale); K, V device pointers to key 0; nk keys (any count, no 64-key alignment needed). Synchronous. */
int pa_cuda_attn_partial(pa_cuda_ctx *ctx, const pa_cuda_shape *shape, const float *Q, float scale, const uint8_t *K,
                         const uint8_t *V, uint32_t nk, float *O, float *m, float *l, void *stream);

/* Host-buffer call (the end-to-end path): Qs_host [n_sets][nkv][rows][hd] f16 is copied to the device, the plan
 * runs, O/m/l are copied back into host buffers; returns after the copies land. Pinned host buffers give full
 * copy bandwidth. */
int pa_cuda_plan_run_host(pa_cuda_plan *plan, const uint16_t *Qs_host, float *O_host, float *m_host, float *l_host,
                          void *stream);

/* LSE merge of n_parts partials Op [n_parts][rows][hd], mp/lp [n_parts][rows] (device) into O [rows][hd], m, l.
 * fold = 1: (O, m, l) already hold a partial, folded in as one more part (merge_partial / pa_merge_big fold). */
int pa_cuda_merge(pa_cuda_ctx *ctx, uint32_t hd, uint64_t rows, uint32_t n_parts, const float *Op, const float *mp,
                  const float *lp, float *O, float *m, float *l, int fold, void *stream);
/* The same merge over partials packed back to back as one all-gather of each part's (O, m, l) delivers them:
 * part c = packed + c * rows*(hd+2): O [rows][hd], then m [rows], then l [rows]. This folds the N position shards of
 * a multi-GPU call (one process per GPU, the partials exchanged with a single NCCL all-gather), generalising the
 * Mac + phone and two-phone split (docs/TWO-PHONES.md:14-18). */
int pa_cuda_merge_gathered(pa_cuda_ctx *ctx, uint32_t hd, uint64_t rows, uint32_t n_parts, const float *packed,
                           float *O, float *m, float *l, int fold, void *stream);
/* ---- position shards over NCCL, in one call: one process per GPU, rank r holding a contiguous position range of every
 * layer (the N-GPU generalisation of the Mac + phone and two-phone split, docs/TWO-PHONES.md:14-18). NCCL is opened
 * (dlopen of libnccl.so.2) on first use; these calls fail with PA_CUDA_ENCCL when it cannot be.
 * pa_cuda_nccl_unique_id: on one rank, the id (`bytes` >= 128) that every rank then passes to
 * pa_cuda_nccl_comm_create, which returns a communicator over the context's device (an opaque handle that wraps an
 * ncclComm_t; destroyed with pa_cuda_nccl_comm_destroy, also after an abort). */
int pa_cuda_nccl_unique_id(void *id, size_t bytes);
int pa_cuda_nccl_comm_create(pa_cuda_ctx *ctx, const void *id, int rank, int world, void **comm);
void pa_cuda_nccl_comm_destroy(void *comm);
/* Runs this rank's plan (its shard's segments) into a packed (O, m, l), exchanges the ranks' partials on `stream`, and
 * folds them by log-sum-exp into O, m, l, identical on every rank. Every rank calls it, in the same order, with plans of
 * the same n_sets and shape, and the same exchange settings. The exchange (pa_cuda_set_shard_exchange):
 *   peer stores: the merge of this rank's chunk partials stores its rows straight into every rank's receive buffer over
 *     NVLink (buffers mapped into every rank with CUDA IPC, set up collectively by the first such call) and counts
 *     them in on a per-source counter there; each rank's fold waits (bounded by pa_cuda_set_timeout_ns: a missing
 *     rank's partial makes pa_cuda_status report PA_CUDA_ETIMEOUT) until every rank's rows are in, then merges. No
 *     NCCL launch on the call's path. The choice by size below 8 MiB of partial per rank (decode, verify); when CUDA
 *     IPC is not available on every rank, all ranks use the all-gather instead.
 *   all-gather: one ncclAllGather of every rank's packed (O, m, l), then the fold (pa_cuda_merge_gathered): each rank
 *     receives N-1 partials. The choice by size for large partials on 2 ranks.
 *   all-reduce: the rows' maxima over the ranks (ncclAllReduce MAX straight into m), each rank's (O, l) moved to them,
 *     then summed (ncclAllReduce SUM into O and l): ~2(N-1)/N of a partial per rank. The choice by size from 8 MiB of
 *     partial per rank with more than 2 ranks (prefill).
 * Set groups (pa_cuda_set_shard_groups): the plan's output sets are split into G contiguous groups; group g's exchange
 * runs on a second stream while the kernels of group g+1 run (by size: 8 groups from 64 MiB of partial per rank).
 * Asynchronous unless a bound is set (pa_cuda_set_shard_timeout_ms); the packed and gathered buffers are the context's
 * own (grown as needed). */
int pa_cuda_shard_attn_allgather_merge(pa_cuda_plan *plan, const uint16_t *Qs, void *comm, float *O, float *m, float *l,
                                       void *stream);
/* Exchange of pa_cuda_shard_attn_allgather_merge for calls made afterwards: 0 = by size (default), 1 = all-gather and
 * fold, 2 = max / sum all-reduces, 3 = peer stores (set groups do not apply). */
void pa_cuda_set_shard_exchange(pa_cuda_ctx *ctx, int mode);
/* The exchange (1, 2 or 3) and set groups the last pa_cuda_shard_attn_allgather_merge of this context used. */
void pa_cuda_shard_last(const pa_cuda_ctx *ctx, int *exchange, int *groups);
/* Output-set groups of pa_cuda_shard_attn_allgather_merge whose exchange overlaps the next group's kernels: 0 = by size
 * (default), 1 = no overlap, G > 1 = G groups (at most n_sets). */
void pa_cuda_set_shard_groups(pa_cuda_ctx *ctx, int groups);
/* Bound on the shard exchange (the B200 counterpart of the client's bounded reply wait, phone-attn/phone-attn.h:796-820):
 * with ms > 0, pa_cuda_shard_attn_allgather_merge returns only once its work on the stream has finished, polling the
 * stream and ncclCommGetAsyncError. On an NCCL error, or when ms pass first (a rank that left or stalled keeps the
 * collective waiting), it aborts the communicator (ncclCommAbort: the collectives in flight return and the stream
 * drains) and returns PA_CUDA_ENCCL or PA_CUDA_ETIMEOUT; O, m and l are then undefined and the communicator fails every
 * later call (destroy it and create a new one). 0 = asynchronous (default). */
void pa_cuda_set_shard_timeout_ms(pa_cuda_ctx *ctx, uint32_t ms);
/* The same bounded wait for callers of the asynchronous mode: waits for the work queued on `stream` (NULL = the
 * context's stream), polling NCCL's asynchronous error, and aborts the communicator on an error or after timeout_ms
 * (0 = no bound). */
int pa_cuda_nccl_wait(pa_cuda_ctx *ctx, void *comm, void *stream, uint32_t timeout_ms);
/* O/l -> f16 Oh, lse = m + log l (device) */
int pa_cuda_normalize(pa_cuda_ctx *ctx, uint32_t hd, uint64_t rows, const float *O, const float *m, const float *l,
                      uint16_t *Oh, float *lse, void *stream);
/* The host's co-attention fold (phone-attn/phone-attn.h:18-20): a normalised reply row (f16 Oh = O/l, lse = m + log l,
 * as ATTN returns it) is re-expanded as the part (O = Oh, m = lse, l = 1) and merged into the unnormalised partial in
 * (O, m, l) with merge_partial's rule (phone-attn/phone-attn.h:231-239): rows with lse = -inf add nothing, rows whose
 * l <= 0 take the reply. Device pointers; Oh [rows][hd], lse [rows]. */
int pa_cuda_fold_reply(pa_cuda_ctx *ctx, uint32_t hd, uint64_t rows, const uint16_t *Oh, const float *lse, float *O,
                       float *m, float *l, void *stream);
/* Qs = f16(Q * scale) for n values (device) */
int pa_cuda_scale_q(pa_cuda_ctx *ctx, const float *Q, float scale, uint64_t n, uint16_t *Qs, void *stream);

/* ---- pa::engine (phone-attn/phone-attn.h:166-183) */
int pa_cuda_alloc_page(pa_cuda_ctx *ctx, size_t bytes, pa_cuda_page *p);
void pa_cuda_free_page(pa_cuda_ctx *ctx, pa_cuda_page *p);
/* Start the partial over n_pages pages (nkeys[i] keys each) for ng groups of 48 query rows per KV head:
 * Qs_host = f16(q*scale) [ng][nkv][48][hd] (phone-attn/phone-attn.h:170-172). ntok (1..8) for ng == 1: the group's
 * real tokens; rows r = g*8 + t with t >= ntok are zero and come back as empty partials (m = -inf, l = 0), as
 * pa_merge_big's ntok packing (phone-attn/pa-metal.mm:505-509). shape->rows is ignored (48). Asynchronous. */
int pa_cuda_begin(pa_cuda_ctx *ctx, const pa_cuda_page *pages, const uint32_t *nkeys, int n_pages,
                  const uint16_t *Qs_host, const pa_cuda_shape *shape, int ng, int ntok);
/* Wait for the call begun last; O [ng][nkv*48][hd], m, l [ng][nkv*48] (host). Returns the milliseconds from begin to
 * completion, or -1 on failure with m = -inf, l = 0 (phone-attn/pa-metal.mm:928-937). */
double pa_cuda_end(pa_cuda_ctx *ctx, float *O, float *m, float *l);
/* GPU execution time of the last completed begin/end call (CUDA events), ms */
double pa_cuda_exec_ms(const pa_cuda_ctx *ctx);
/* engine::arm (phone-attn/phone-attn.h:179-182): the next one-group call will likely be this one (the next layer, same
 * split and tokens). Prepares it: the call's plan (kept per call shape, as every begin keeps its own) and a CUDA graph
 * of the whole call (Q upload, kernels, readback). The graph stays with the cached plan: every later begin with the
 * same pages, key counts, geometry and ntok packs Q and launches it; any other begin runs as usual (pa-metal.mm:716-765
 * encodes and parks a one-shot command buffer instead). Call between end and the next begin, from the thread that calls
 * begin. Advisory: an error leaves begin unaffected. */
int pa_cuda_arm(pa_cuda_ctx *ctx, const pa_cuda_page *pages, const uint32_t *nkeys, int n_pages, const pa_cuda_shape *shape,
                int ntok);
/* number of begin calls served by an armed graph */
uint64_t pa_cuda_graph_calls(const pa_cuda_ctx *ctx);

/* ---- allocation-free call (no counterpart in the reference: an addition of this library)
 * For callers that cannot allocate device memory: a host runtime that owns every device allocation itself (a fixed
 * memory pool, an inference server that reserves the GPU's memory up front), or code running where cudaMalloc is not
 * allowed, cannot create a context (pa_cuda_create allocates) or a plan (plans own scratch). This entry point runs the
 * split-K kernel and the merge for one segment (as pa_cuda_attn with one set and one segment) using a fixed 16 MiB
 * device array compiled into the library instead of allocated scratch; it calls no cudaMalloc, cudaFree or other
 * allocating routine. The caller still passes Qs (f16(q*scale) [nkv][rows][hd]), K, V (device) and O, m, l.
 *   Limit: one chunk partial, nkv * rows * (hd + 2) * 4 bytes, must fit the 16 MiB array (up to 2048 chunks are used);
 *   a larger shape returns PA_CUDA_EUNSUPPORTED with the reason in *why (a static string; why may be null).
 *   Set-up: the first call on a device looks the array's device address up (cudaGetSymbolAddress, with that device
 *   current); make that first call before any stream capture. Under CUDA's lazy module loading (the default) that first
 *   call is also when the library's kernels and the 16 MiB array are loaded onto the device: a host that reserves all
 *   free device memory for its own pool makes the first call before reserving it, or leaves ~16 MiB plus the module
 *   free. Every GPU that loads the library holds the array until the process exits. The address is kept per device for
 *   the life of the process, so a process that calls cudaDeviceReset does not use this entry point afterwards.
 *   Sharing: all calls on a device share the one array and it keeps the last call's contents (each call rewrites what
 *   it reads); calls that overlap on the GPU (other streams, other host threads) race and must be serialised.
 *   The call returns after the stream has synchronised: PA_CUDA_OK, or PA_CUDA_ETIMEOUT if a bounded wait ran out.
 *   stream: a cudaStream_t (NULL: the default stream). */
int pa_cuda_attn_noalloc(const pa_cuda_shape *shape, const uint16_t *Qs, const uint8_t *K, const uint8_t *V, uint32_t nk,
                         float *O, float *m, float *l, void *stream, const char **why);

#ifdef __cplusplus
}
#endif
