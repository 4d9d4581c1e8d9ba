// Allocation-free entry point for split-KV paged decode attention.
//
// This entry point has no counterpart in the reference (MIT-RLX/rlx-models);
// it is an addition of this library.
//
// Who it is for: callers that cannot call cudaMalloc (or any allocating
// routine) at the point where they run attention. Typical cases are host
// applications that link this library from plain C and own every byte of
// device memory themselves under a fixed budget decided at start-up, plugin
// hosts whose custom-op interface forbids allocation, and latency-critical
// loops that cannot afford cudaMalloc's implicit device synchronisation or its
// chance of failing at run time. They still pass all inputs and outputs; the
// only memory this call needs beyond those - the per-split partial results of
// split-KV attention - lives in a fixed, file-scope device array compiled
// into the library.
//
// Scratch capacity: B * Hq * splits * (head_dim + 2) floats must not exceed
// B200_NOALLOC_SCRATCH_FLOATS (1 << 20 floats = 4 MiB). Larger requests are
// rejected with B200_NOALLOC_ERR_SCRATCH before anything is launched. Every
// GPU that loads the library holds these 4 MiB until the process exits.
//
// Set-up: the first call on a device (with that device current) looks up the
// device address of the scratch array with cudaGetSymbolAddress and sets the
// kernel's shared-memory attribute; make that first call before any stream
// capture. Later calls on the same device do no set-up. The looked-up address
// is cached per device ordinal for the life of the process: a caller that
// resets the device (cudaDeviceReset) or destroys and recreates its primary
// context must not call this entry point afterwards in the same process.
//
// Sharing: all calls on a device share the one scratch array, which keeps the
// previous call's contents. Every slot a call reads is written earlier in the
// same call, so nothing has to start at zero. Calls whose executions overlap on
// the GPU (different streams without ordering between them) race on the array
// and give wrong results; order such calls on one stream or with events.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_NOALLOC_SCRATCH_FLOATS (1 << 20)

enum {
  B200_NOALLOC_OK = 0,
  B200_NOALLOC_ERR_ARGS = 1,     // unsupported shape / null pointer / splits < 1
  B200_NOALLOC_ERR_SCRATCH = 2,  // B * Hq * splits * (D + 2) > B200_NOALLOC_SCRATCH_FLOATS
  B200_NOALLOC_ERR_SETUP = 3,    // cudaGetSymbolAddress / attribute set-up failed
  B200_NOALLOC_ERR_TMA = 4,      // tensor-map encoding failed
  B200_NOALLOC_ERR_LAUNCH = 5,   // one of this call's own kernel launches failed
};

// q: [B, Hq, D] bf16; k_cache / v_cache: [num_blocks, Hkv, 16, D] bf16;
// block_tables: [B, max_blocks] int32; ctx_lens: [B] int32 (kv length incl.
// the new token; each must be <= 16 * max_blocks: a longer one is clamped to
// the table and flagged in `status` as a bounds error); out: [B, Hq, D] bf16;
// sinks: [Hq] fp32 or NULL; window: 0 for full attention; splits >= 1 (the KV range of each sequence is cut into
// `splits` parts whose partials meet in the scratch array); status: optional
// device int32[4] error word (NULL to skip); stream: a cudaStream_t.
// D must be 64 or 128 and Hq / Hkv <= 16. Returns a B200_NOALLOC_* code.
__attribute__((visibility("default"))) int b200_decode_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, int64_t num_blocks, const int32_t* block_tables,
    int max_blocks, const int32_t* ctx_lens, void* out, const float* sinks, int window, int B, int Hq, int Hkv,
    int D, float scale, int splits, int* status, void* stream);

#ifdef __cplusplus
}
#endif
