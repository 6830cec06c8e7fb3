// pa_cuda_engine.h - pa::cuda_engine: the reference's GPU-engine interface (pa::engine, phone-attn/phone-attn.h:166-183)
// implemented over libpacuda.so's C ABI (include/pa_cuda.h), in the place of the Metal engine
// (phone-attn/pa-metal.mm:532-996).
//
// Include it after phone-attn.h, as pa-tool.cpp includes pa-metal.mm (phone-attn/pa-tool.cpp:7-10), and hand an
// instance to pa::server:
//     auto * gpu = new pa::cuda_engine();
//     if (!gpu->init(0)) { fprintf(stderr, "CUDA engine off: %s\n", gpu->error.c_str()); delete gpu; gpu = nullptr; }
//     pa::server srv(&st, log, threads, gpu);
// Link with -lpacuda. With an engine present and no SME2, pa::server gives the engine every page
// (phone-attn/phone-attn.h:588), so the server needs no change.
//
// Contract kept from the reference engine:
//   alloc_page/free_page : page memory the host writes (pa::server's APPEND memcpy's rows into it) and the GPU reads
//                          without a copy: CUDA managed memory, preferred on the device, prefetched by begin().
//   begin                : asynchronous; Qs = f16(q*scale) [ng][nkv][48][256]; one-group calls pack only the
//                          ntok_hint real tokens' rows (phone-attn/pa-metal.mm:627-646).
//   end                  : waits; unnormalised O [ng][nkv*48][256], m, l; -1 and m = -inf, l = 0 on failure
//                          (phone-attn/pa-metal.mm:928-937).
//   page formats         : whatever the server's store_cfg() says (phone-attn/phone-attn.h:298-302): Q8_0 and Q4_0
//                          rows as received, or f16 rows (is_q8 == 0, store_f16), all on the split-K kernel; calls of
//                          >= 32 rows per KV head with quantised rows (ATTN_BIG, multi-token ATTN) run on the tcgen05
//                          CTA-pair kernel at the server's HD 256.
#pragma once
#include <cstdlib>
#include <string>
#include <vector>

#include "pa_cuda.h"

namespace pa {

class cuda_engine : public engine {
public:
    std::string error;

    bool init(int device = 0) {
        if (!pa_cuda_available()) { error = "no sm_100 CUDA device, or libpacuda.so's kernels do not load"; return false; }
        if (pa_cuda_create(device, &ctx_) != PA_CUDA_OK) { error = "pa_cuda_create failed"; ctx_ = nullptr; return false; }
        return true;
    }
    ~cuda_engine() override { if (ctx_) pa_cuda_destroy(ctx_); }

    bool alloc_page(size_t bytes, page & p) override {
        pa_cuda_page cp{};
        if (pa_cuda_alloc_page(ctx_, bytes, &cp) != PA_CUDA_OK) { error = pa_cuda_last_error(ctx_); return false; }
        p.k = cp.k; p.v = cp.v; p.hk = cp.hk; p.hv = cp.hv;
        return true;
    }
    void free_page(page & p) override {
        pa_cuda_page cp{p.k, p.v, p.hk, p.hv};
        pa_cuda_free_page(ctx_, &cp);
        p = page();
    }
    bool begin(const page * pages, const uint32_t * nkeys, int n_pages, const uint16_t * Qs, const config_req & cfg,
               int ng = 1) override {
        std::vector<pa_cuda_page> cp((size_t) n_pages);
        for (int i = 0; i < n_pages; i++) cp[(size_t) i] = pa_cuda_page{pages[i].k, pages[i].v, pages[i].hk, pages[i].hv};
        const pa_cuda_shape sh{(uint32_t) HD, cfg.n_head_kv, (uint32_t) NR, cfg.is_q8, cfg.rs, cfg.hb};
        ng_ = ng;
        rows_ = (int) cfg.n_head_kv * NR;
        const int rc = pa_cuda_begin(ctx_, cp.data(), nkeys, n_pages, Qs, &sh, ng, ng == 1 ? ntok_hint : 8);
        if (rc != PA_CUDA_OK) { error = pa_cuda_last_error(ctx_); return false; }
        calls_++;
        return true;
    }
    double end(float * O, float * m, float * l) override {
        const double ms = pa_cuda_end(ctx_, O, m, l);
        if (ms < 0) error = pa_cuda_last_error(ctx_);
        return ms;
    }
    double exec_ms() const override { return pa_cuda_exec_ms(ctx_); }
    // the server's hint that the next call is this one (phone-attn/phone-attn.h:686-697): its plan and a CUDA graph of
    // the whole call are prepared now, off the next call's critical path (PA_CUDA_ARM=0 turns it off)
    void arm(const page * pages, const uint32_t * nkeys, int n_pages, const config_req & cfg, int ntok) override {
        static const bool on = !getenv("PA_CUDA_ARM") || atoi(getenv("PA_CUDA_ARM")) != 0;
        if (!on || n_pages <= 0) return;
        std::vector<pa_cuda_page> cp((size_t) n_pages);
        for (int i = 0; i < n_pages; i++) cp[(size_t) i] = pa_cuda_page{pages[i].k, pages[i].v, pages[i].hk, pages[i].hv};
        const pa_cuda_shape sh{(uint32_t) HD, cfg.n_head_kv, (uint32_t) NR, cfg.is_q8, cfg.rs, cfg.hb};
        if (pa_cuda_arm(ctx_, cp.data(), nkeys, n_pages, &sh, ntok) == PA_CUDA_OK) armed_++;
    }
    std::string describe() override {
        char b[224];
        snprintf(b, sizeof b, "engine=pa-cuda calls=%llu armed=%llu graph_calls=%llu last_gpu_exec_ms=%.3f launches=%llu",
                 (unsigned long long) calls_, (unsigned long long) armed_,
                 (unsigned long long) pa_cuda_graph_calls(ctx_), pa_cuda_exec_ms(ctx_),
                 (unsigned long long) pa_cuda_launch_count(ctx_));
        return b;
    }

private:
    pa_cuda_ctx * ctx_ = nullptr;
    int ng_ = 1, rows_ = 0;
    unsigned long long calls_ = 0, armed_ = 0;
};

}  // namespace pa
