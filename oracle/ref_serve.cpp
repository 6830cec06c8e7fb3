// ref_serve.cpp - the reference's own phone-attn server (pa::server from phone-attn/phone-attn.h, unmodified) with
// a pa::engine plugged in, as `pa-tool serve` does with PA_GPU=1 (phone-attn/pa-tool.cpp:55-82).
// TEST INFRASTRUCTURE ONLY, built into oracle/_ref/ by oracle/Makefile when the reference tree is present:
//   pa-serve-oracle : engine = the oracle's fp32 block-online restatement (oracle/pa_oracle.c). Running the
//                     reference's `pa-tool test` against it checks the oracle with the reference's own fp64 gate
//                     (phone-attn/pa-tool.cpp:150-173) through the reference's server (attn_core, merge, normalise).
//   pa-serve-cuda   : engine = pa::cuda_engine (backburner_b200/csrc/pa_cuda_engine.h) over libpacuda.so: the
//                     CUDA path behind the unchanged wire protocol (-DPA_SERVE_CUDA).
// usage: pa-serve [port] [threads]
#include "phone-attn.h"
#include "sme_stub.h"

#ifdef PA_SERVE_CUDA
#include "pa_cuda_engine.h"
#else
#include "pa_oracle.h"
#endif

#include <cstdio>
#include <cstdlib>
#include <vector>

#ifndef PA_SERVE_CUDA
namespace {
// pa::engine over host memory: begin() computes every page with the oracle and folds the pages with the reference's
// merge_partial; end() hands the result over.
struct oracle_engine : pa::engine {
    std::vector<float> O_, m_, l_;
    bool alloc_page(size_t bytes, pa::page & p) override {
        const size_t n = (bytes + 16383) / 16384 * 16384;
        p.k = (uint8_t *) aligned_alloc(16384, n);
        p.v = (uint8_t *) aligned_alloc(16384, n);
        return p.k && p.v;
    }
    void free_page(pa::page & p) override { free(p.k); free(p.v); p = pa::page(); }
    bool begin(const pa::page * pages, const uint32_t * nkeys, int n_pages, const uint16_t * Qs, const pa::config_req & cfg,
               int ng) override {
        const size_t rows = (size_t) cfg.n_head_kv * pa::NR, qn = rows * pa::HD;
        O_.assign((size_t) ng * qn, 0.0f); m_.assign((size_t) ng * rows, -INFINITY); l_.assign((size_t) ng * rows, 0.0f);
        orc_shape sh = { pa::HD, (int) cfg.n_head_kv, pa::NR, (int) cfg.is_q8, cfg.rs, cfg.hb };
        std::vector<float> O2(qn), m2(rows), l2(rows);
        for (int g = 0; g < ng; g++) {
            for (int i = 0; i < n_pages; i++) {
                if (orc_partial_f32_mt(&sh, Qs + (size_t) g * qn, pages[i].k, pages[i].v, nkeys[i], 4, 1024, O2.data(), m2.data(),
                                       l2.data()) != 0) return false;
                pa::merge_partial(O_.data() + (size_t) g * qn, m_.data() + (size_t) g * rows, l_.data() + (size_t) g * rows,
                                  O2.data(), m2.data(), l2.data(), rows);
            }
        }
        return true;
    }
    double end(float * O, float * m, float * l) override {
        std::copy(O_.begin(), O_.end(), O); std::copy(m_.begin(), m_.end(), m); std::copy(l_.begin(), l_.end(), l);
        return 0.0;
    }
    std::string describe() override { return "engine=oracle-fp32"; }
};
}  // namespace
#endif

int main(int argc, char ** argv) {
    const int port = argc > 1 ? atoi(argv[1]) : pa::DEFAULT_PORT;
    const int thr = argc > 2 ? atoi(argv[2]) : 2;
    pa::status st;
#ifdef PA_SERVE_CUDA
    auto * eng = new pa::cuda_engine();
    if (!eng->init(getenv("PA_CUDA_DEVICE") ? atoi(getenv("PA_CUDA_DEVICE")) : 0)) {
        fprintf(stderr, "CUDA engine off: %s\n", eng->error.c_str());
        return 1;
    }
#else
    auto * eng = new oracle_engine();
#endif
    pa::server srv(&st, [](const std::string & s) { fprintf(stderr, "%s\n", s.c_str()); }, thr, eng);
    fprintf(stderr, "%s\n", srv.serve(port).c_str());
    return 1;
}
