// ref_client.cpp - TEST INFRASTRUCTURE ONLY: the reference's own pa::client (phone-attn/phone-attn.h:741-842, unmodified)
// drives a pa::server through the store protocol around the attention calls: CONFIG, APPEND, ATTN, TRUNCATE, ATTN,
// FETCH, APPEND (new rows over the truncated range), ATTN, FETCH, STATS (server: phone-attn/phone-attn.h:388-482; client:
// :758-776). Every ATTN reply is checked against the oracle's fp64 partial (oracle/pa_oracle.c) over exactly the keys the
// server holds at that point, normalised as attn_core does (O/l, lse = m + log l), with pa-tool's metrics and 5e-3 gate
// (phone-attn/pa-tool.cpp:150-173); every FETCH is compared byte for byte with the rows appended at those positions.
// Built into oracle/_ref/ by oracle/Makefile; run against oracle/_ref/pa-serve-cuda by tests/test_pa_tool_gpu.py.
// usage: pa-client-check host port [quant: 1 = q8_0 (default), 2 = q4_0]
#include "phone-attn.h"
#include "sme_stub.h"
#include "pa_oracle.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

namespace {

constexpr int NKV = 4, NL = 2;
constexpr float SCALE = 1.0f / 16;
int g_fail = 0;

struct Store {   // what the server should hold for one layer
    int quant = 1;
    size_t rs = 0;
    std::vector<uint8_t> K, V;
    uint32_t n = 0;
};

void rows(Store & s, uint32_t pos0, uint32_t n, uint64_t seed) {
    s.K.resize((size_t) (pos0 + n) * s.rs);
    s.V.resize((size_t) (pos0 + n) * s.rs);
    uint64_t st = seed;
    for (uint32_t j = pos0; j < pos0 + n; j++) {
        if (s.quant == ORC_Q4_0) {
            orc_pt_make_q4_row(&s.K[(size_t) j * s.rs], NKV, 1.5f, &st);
            orc_pt_make_q4_row(&s.V[(size_t) j * s.rs], NKV, 1.0f, &st);
        } else {
            orc_pt_make_q8_row(&s.K[(size_t) j * s.rs], NKV, 1.5f, &st);
            orc_pt_make_q8_row(&s.V[(size_t) j * s.rs], NKV, 1.0f, &st);
        }
    }
}

bool append(pa::client & c, int layer, Store & s, uint32_t pos0, uint32_t n, uint64_t seed) {
    rows(s, pos0, n, seed);
    for (uint32_t p0 = pos0; p0 < pos0 + n; p0 += pa::PAGE) {
        const uint32_t k = std::min<uint32_t>(pa::PAGE, pos0 + n - p0);
        if (!c.append(layer, p0, k, &s.K[(size_t) p0 * s.rs], &s.V[(size_t) p0 * s.rs], s.rs)) {
            printf("append layer %d pos %u: %s\n", layer, p0, c.last_err.c_str());
            return false;
        }
    }
    s.n = pos0 + n;
    return true;
}

// one ATTN call of ntok tokens over all held keys of `layer`, checked against the fp64 oracle over s.K/V[0, s.n)
bool attn_check(pa::client & c, int layer, const Store & s, int ntok, const char * what) {
    const size_t qn = (size_t) NKV * pa::NR * pa::HD;
    std::vector<uint16_t> Q(qn), O(qn), Qs(qn);
    std::vector<float> lse(qn / pa::HD);
    uint64_t st = 0x9E3779B97F4A7C15ull ^ (uint64_t) (s.n * 31 + ntok);
    for (size_t i = 0; i < qn; i++) {
        Q[i] = ((i / pa::HD) % 8 < (size_t) ntok) ? orc_f2h(orc_lcg_frand(&st) * 1.7f) : 0;
        Qs[i] = orc_f2h(orc_h2f(Q[i]) * SCALE);   // attn_core's f16(q * scale) (phone-attn/phone-attn.h:595-599)
    }
    pa::attn_rep rep;
    if (!c.attn(layer, ntok, 0, SCALE, Q.data(), qn, O.data(), lse.data(), rep)) {
        printf("%s: attn: %s\n", what, c.last_err.c_str());
        return false;
    }
    const orc_shape sh = {pa::HD, NKV, pa::NR, s.quant, s.rs, s.rs / NKV};
    std::vector<double> Or(qn), mr(qn / pa::HD), lr(qn / pa::HD);
    orc_partial_f64(&sh, Qs.data(), s.K.data(), s.V.data(), s.n, Or.data(), mr.data(), lr.data());
    double eo = 0, el = 0;
    for (size_t r = 0; r < qn / pa::HD; r++) {
        if ((int) ((r % pa::NR) % 8) >= ntok) continue;
        double omax = 1e-30;
        for (int d = 0; d < pa::HD; d++) omax = std::max(omax, std::fabs(Or[r * pa::HD + d] / lr[r]));
        for (int d = 0; d < pa::HD; d++)
            eo = std::max(eo, std::fabs(orc_h2f(O[r * pa::HD + d]) - Or[r * pa::HD + d] / lr[r]) / omax);
        el = std::max(el, std::fabs(lse[r] - (mr[r] + std::log(lr[r]))));
    }
    const bool ok = rep.nk == s.n && eo < 5e-3 && el < 5e-3;
    printf("%s (layer %d, %u keys held, %d tokens, reply nk %u): max|O - ref|/max|ref| = %.2e  max|lse - ref| = %.2e -> %s\n",
           what, layer, s.n, ntok, rep.nk, eo, el, ok ? "PASS" : "FAIL");
    if (!ok) g_fail++;
    return true;
}

bool fetch_check(pa::client & c, int layer, const Store & s, uint32_t pos0, uint32_t n, const char * what) {
    std::vector<uint8_t> got((size_t) n * s.rs);
    bool ok = true;
    for (uint32_t which = 0; which < 2; which++) {
        if (!c.fetch(layer, pos0, n, which, got.data(), s.rs)) {
            printf("%s: fetch: %s\n", what, c.last_err.c_str());
            return false;
        }
        const uint8_t * want = (which ? s.V.data() : s.K.data()) + (size_t) pos0 * s.rs;
        size_t bad = 0;
        for (size_t i = 0; i < got.size(); i++) bad += got[i] != want[i];
        printf("%s (layer %d, %s rows [%u, %u)): %zu bytes differ -> %s\n", what, layer, which ? "V" : "K", pos0, pos0 + n,
               bad, bad ? "FAIL" : "PASS");
        ok = ok && bad == 0;
    }
    if (!ok) g_fail++;
    return true;
}

}  // namespace

int main(int argc, char ** argv) {
    if (argc < 3) { fprintf(stderr, "usage: pa-client-check host port [quant]\n"); return 2; }
    const int quant = argc > 3 ? atoi(argv[3]) : 1;
    pa::client c;
    if (!c.connect(argv[1], atoi(argv[2]))) { printf("connect: %s\n", c.last_err.c_str()); return 1; }
    pa::hello_rep hr;
    if (!c.hello(hr)) { printf("hello: %s\n", c.last_err.c_str()); return 1; }
    const uint32_t hb = quant == ORC_Q4_0 ? 144 : 272, rs = NKV * hb;
    const pa::config_req cfg = {NL, NKV, rs, hb, (uint32_t) quant, 1, 1, 0, 1024, 0, 0};
    if (!c.config(cfg)) { printf("config: %s\n", c.last_err.c_str()); return 1; }
    Store s[NL];
    for (int L = 0; L < NL; L++) { s[L].quant = quant; s[L].rs = rs; }
    // 12,800 keys per layer: three full pages and one partial page
    for (int L = 0; L < NL; L++) if (!append(c, L, s[L], 0, 12800, 1000 + L)) return 1;
    if (!attn_check(c, 0, s[0], 8, "ATTN after APPEND") || !attn_check(c, 1, s[1], 1, "ATTN after APPEND")) return 1;
    // rewind into the middle of page 1 (the pages past it are dropped), then read back rows the GPU has read
    if (!c.truncate(4992)) { printf("truncate: %s\n", c.last_err.c_str()); return 1; }
    for (int L = 0; L < NL; L++) { s[L].n = 4992; s[L].K.resize((size_t) 4992 * rs); s[L].V.resize((size_t) 4992 * rs); }
    if (!attn_check(c, 0, s[0], 8, "ATTN after TRUNCATE") || !attn_check(c, 1, s[1], 1, "ATTN after TRUNCATE")) return 1;
    if (!fetch_check(c, 0, s[0], 0, 4992, "FETCH after TRUNCATE") || !fetch_check(c, 1, s[1], 4000, 992, "FETCH after TRUNCATE"))
        return 1;
    // new rows over the truncated range, up to the same 12,800 keys as before: the page the truncation cut into is
    // rewritten at the same key count, and the dropped pages come back as new ones
    for (int L = 0; L < NL; L++) if (!append(c, L, s[L], 4992, 7808, 2000 + L)) return 1;
    if (!attn_check(c, 0, s[0], 8, "ATTN after re-APPEND") || !attn_check(c, 1, s[1], 8, "ATTN after re-APPEND")) return 1;
    if (!fetch_check(c, 0, s[0], 4096, 8704, "FETCH after re-APPEND") || !fetch_check(c, 1, s[1], 0, 12800, "FETCH after re-APPEND"))
        return 1;
    // a rewind to a page boundary and a short APPEND
    if (!c.truncate(8192)) { printf("truncate: %s\n", c.last_err.c_str()); return 1; }
    for (int L = 0; L < NL; L++) { s[L].K.resize((size_t) 8192 * rs); s[L].V.resize((size_t) 8192 * rs); s[L].n = 8192; }
    for (int L = 0; L < NL; L++) if (!append(c, L, s[L], 8192, 1344, 3000 + L)) return 1;
    if (!attn_check(c, 0, s[0], 1, "ATTN after TRUNCATE to a page boundary") ||
        !attn_check(c, 1, s[1], 8, "ATTN after TRUNCATE to a page boundary")) return 1;
    if (!fetch_check(c, 0, s[0], 8000, 1536, "FETCH across the page boundary")) return 1;
    const std::string st = c.stats();
    printf("peer stats: %s\n", st.c_str());
    if (st.find("engine=") == std::string::npos) { printf("STATS without the engine's description -> FAIL\n"); g_fail++; }
    printf(g_fail ? "%d FAILED\n" : "ALL PASS\n", g_fail);
    return g_fail ? 1 : 0;
}
