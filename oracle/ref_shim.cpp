// ref_shim.cpp - exposes the reference's own test-data generators, dequantiser, f16 conversions and host merge
// (compiled from the reference sources where they lie) through a C ABI, so the tests can pin the oracle
// restatement against the reference bit for bit. TEST INFRASTRUCTURE ONLY; built into oracle/_ref/ by
// oracle/Makefile, only when the reference tree is present.
//
// The reference's pa-tool.cpp is included whole, with its main() renamed, so its file-static helpers
// (frand, make_q8_row, make_q4_row, deq; phone-attn/pa-tool.cpp:16-51) are callable from here.
// x86 shims: __fp16 -> _Float16, TARGET_OS_IPHONE=0, __builtin_arm_yield() -> no-op (passed by the Makefile).
#define main pa_tool_main
#include "pa-tool.cpp"
#undef main

#include "sme_stub.h"

extern "C" {

// pa-tool.cpp:16-17: n values of the LCG from state `seed` (the reference's default state is 0x9e3779b97f4a7c15)
void ref_frand_seq(uint64_t seed, float * out, int n) {
    g_s = seed;
    for (int i = 0; i < n; i++) out[i] = frand();
}

// pa-tool.cpp:20-40: n rows of nkv heads (HD 256) from LCG state `seed`; q4 != 0 selects make_q4_row
void ref_make_rows(uint64_t seed, int q4, int n, int nkv, float amp, uint8_t * out) {
    g_s = seed;
    const size_t rs = (size_t) nkv * (q4 ? 144 : 272);
    for (int j = 0; j < n; j++) {
        if (q4) make_q4_row(out + (size_t) j * rs, nkv, amp);
        else    make_q8_row(out + (size_t) j * rs, nkv, amp);
    }
}

// pa-tool.cpp:41-51: the exact dequantised value of head h, dim d of one row
float ref_deq(const uint8_t * row, int q4, int h, int d) {
    g_q4 = q4;
    return deq(row, h, d);
}

// phone-attn.h:120-121
uint16_t ref_f2h(float f) { return pa::f2h(f); }
float    ref_h2f(uint16_t h) { return pa::h2f(h); }

// phone-attn.h:231-239 (rows of HD = 256)
void ref_merge_partial(float * O, float * m, float * l, const float * O2, const float * m2, const float * l2, size_t rows) {
    pa::merge_partial(O, m, l, O2, m2, l2, rows);
}

int ref_hd(void) { return pa::HD; }
int ref_nr(void) { return pa::NR; }

}
