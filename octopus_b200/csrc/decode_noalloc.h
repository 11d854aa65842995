// Allocation-free paged decode attention: one C entry point.
//
// This entry point has no counterpart in the reference project; it is an addition of
// this library.
//
// Who needs it: code that must not allocate device memory while it runs.  Examples are
// a plugin hosted by another runtime that owns all of the GPU's memory and hands out
// only the buffers it planned, a serving loop whose memory budget is fixed up front so
// that a request can never fail on an out-of-memory allocation halfway through, and a
// latency-critical loop that cannot afford the implicit device synchronisation that
// cudaMalloc / cudaFree can cause.  Those callers can pass their inputs and outputs
// but cannot let the library grab scratch space, which the regular decode path
// (octopus_b200.ops.DecodeAttention) takes from the PyTorch allocator.
//
// What it does: the same split-K decode attention as the regular path (one query row
// per request, keys gathered from a page-size-1 KV cache through per-request slot
// lists, GQA), with its split-K partial results kept in a fixed, file-scope device
// array instead of an allocated buffer.  Nothing is allocated: no cudaMalloc,
// cudaFree or allocating library call happens inside it.
//
// Limits and rules:
//   * The static scratch holds OCTO_NOALLOC_MAX_PARTIAL_FLOATS floats of partial outputs
//     (B * Hq * num_splits * head_dim must not exceed it) and
//     OCTO_NOALLOC_MAX_PARTIAL_ROWS log-normalisers (B * Hq * num_splits must not exceed
//     it); larger calls are rejected with OCTO_NOALLOC_ERR_TOO_LARGE and a message on
//     stderr.  Every GPU on which the library is loaded holds this array (about 8.3 MB)
//     until the process exits.
//   * The first call on a device resolves the array's device address (with that device
//     current) and caches it per device; make that first call before any stream
//     capture begins on that device.
//   * All calls share the one array and it keeps the previous call's contents.  Every
//     partial the combine step reads is written earlier in the same call, so nothing
//     needs clearing, but two calls whose kernels overlap on the GPU (different streams
//     without ordering) race on the scratch and give wrong results: order them.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#define OCTO_NOALLOC_MAX_PARTIAL_FLOATS (2 * 1024 * 1024)
#define OCTO_NOALLOC_MAX_PARTIAL_ROWS (64 * 1024)

#define OCTO_NOALLOC_OK 0
#define OCTO_NOALLOC_ERR_TOO_LARGE (-1)     // sizes exceed the static scratch
#define OCTO_NOALLOC_ERR_UNSUPPORTED (-2)   // head_dim not 64/128, Hq % Hkv != 0, GQA group > 16, or
                                            // misaligned / null pointers or strides (see below)
#define OCTO_NOALLOC_ERR_SETUP (-3)         // the scratch address could not be resolved
#define OCTO_NOALLOC_ERR_LAUNCH (-4)        // a kernel launch failed

#ifdef __cplusplus
extern "C" {
#endif

// o[b, h, :] = softmax(q[b, h, :] . K[slots_b]^T * scale) V[slots_b] for every request b,
// with slots_b = kv_indices[kv_start[b] : kv_start[b] + kv_len[b]].
//   q:       bf16 [B, Hq * head_dim], row stride ldq (elements)
//   k_cache, v_cache: bf16 [slots, Hkv * head_dim] (row stride Hkv * head_dim)
//   kv_start, kv_len: int32 [B];  kv_indices: int32 slot ids
//   o:       bf16 [B, Hq * head_dim], row stride ldo (elements)
//   num_splits: key-range splits per request (1..64); 1 needs no scratch at all
// Alignment: k_cache and v_cache 16-byte aligned; q, o and the int32 tables 4-byte
// aligned; ldq and ldo even and at least Hq * head_dim.  Other inputs are refused with
// OCTO_NOALLOC_ERR_UNSUPPORTED before anything is launched.
// Returns OCTO_NOALLOC_OK or one of the OCTO_NOALLOC_ERR_* codes.  OCTO_NOALLOC_ERR_LAUNCH
// reports a failure of this call's own launches; an error left pending by earlier,
// unrelated work is not cleared here and surfaces at the caller's next error check.
int octo_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, const int32_t* kv_start,
                                  const int32_t* kv_len, const int32_t* kv_indices, void* o, int B, int Hq, int Hkv,
                                  int head_dim, int ldq, int ldo, int num_splits, float scale, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
