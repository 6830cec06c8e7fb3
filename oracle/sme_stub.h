// sme_stub.h - definitions for the reference's SME2 C ABI (phone-attn/phone-attn.h:63-71) on a machine without
// SME2: sme2_available() answers 0, so pa::server never calls the others (phone-attn/phone-attn.h:588-593).
// TEST INFRASTRUCTURE ONLY: lets the reference's server and pa-tool link on x86.
#pragma once
#include <cstddef>
#include <cstdint>

extern "C" {
void * sme_ws_new(void) { return nullptr; }
void   sme_attn_partial(void *, const float *, int, const uint8_t *, const uint8_t *, size_t, int, int, float, int, float *,
                        float *, float *) {}
int    sme2_available(void) { return 0; }
void * sme_pipe_new(int) { return nullptr; }
void   sme_attn_pipe(void **, int, int, const float *, const uint8_t *, const uint8_t *, size_t, size_t, int, int, int,
                     float, float *, float *, float *) {}
}
