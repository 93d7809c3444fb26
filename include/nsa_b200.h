/*
 * nsa_b200.h -- C ABI of the B200 (sm_100a) decode-attention library.
 *
 * Every entry point takes raw device pointers, int64 sizes and a CUDA stream,
 * enqueues its kernels on that stream and returns an int status (NSA_OK = 0).
 * Nothing here allocates device memory: scratch space ("workspace") is passed
 * in by the caller, sized by the matching *_workspace_bytes() query, and must
 * be zero-filled once before its first use (the kernels leave it zeroed again).
 * A workspace must not be shared by launches that can run concurrently.
 *
 * Tensors are dense, row-major ("contiguous" in PyTorch terms), 16-byte
 * aligned.  Attention paths take float16 q / k / v and write float16 o.
 * Shapes follow the reference (ayush-os/numerics-and-sparse-attn):
 *   q, o       [B, H, D]          H = 8 * Hkv (GQA group 8), D = 128
 *   k, v       [B, Hkv, L, D]
 * Grids are derived from the shapes passed in (the reference sized them from
 * module constants), so any batch size and any Hkv are accepted.
 *
 * Errors: argument problems are reported synchronously (NSA_ERR_INVALID,
 * NSA_ERR_ALIGN, NSA_ERR_UNSUPPORTED, NSA_ERR_WORKSPACE) with a message from
 * nsa_last_error_message(); launch failures as NSA_ERR_CUDA.  Kernels never
 * trap: a device-side wait that exceeds its time limit records
 * NSA_ERR_TIMEOUT in a device error word, read (and cleared) by
 * nsa_device_error().
 */
#ifndef NSA_B200_H_
#define NSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* nsa_stream_t; /* == cudaStream_t */

enum {
  NSA_OK = 0,
  NSA_ERR_INVALID = 1,     /* bad shape / argument */
  NSA_ERR_ALIGN = 2,       /* pointer not 16-byte aligned */
  NSA_ERR_UNSUPPORTED = 3, /* shape the kernels do not implement (e.g. D != 128) */
  NSA_ERR_WORKSPACE = 4,   /* workspace missing or too small */
  NSA_ERR_CUDA = 5,        /* CUDA runtime / launch error */
  NSA_ERR_TIMEOUT = 6      /* device-side wait exceeded its limit (device error word) */
};

/* Human-readable name of a status code. */
const char* nsa_error_string(int status);
/* Detail of the last failed call on this host thread ("" if none). */
const char* nsa_last_error_message(void);
/* Synchronize `stream`, then read and clear the device error word of the
 * current device into *code (NSA_OK if no kernel recorded an error). */
int nsa_device_error(int* code, nsa_stream_t stream);
/* Library version string. */
const char* nsa_version(void);

/* ------------------------------------------------------------------ dense
 * Dense causal GQA decode over cache slots [0, seq_len) of a cache holding
 * cache_len slots per (batch, kv-head).
 * Replaces dense_kernel.py:70-82 dense_decode_attention(q, k, v, seq_len,
 * sm_scale) and its kernel dense_kernel.py:21-67 (which requires
 * seq_len == cache_len).  seq_len == 0 yields NaN rows, as the reference's
 * 0/0 does.  Split-K: the (batch*kv-head, 64-token tile) space is divided
 * evenly among persistent CTAs; partial results are merged by a log-sum-exp
 * combine inside the same launch. */
size_t nsa_dense_workspace_bytes(int64_t batch, int64_t n_kv_heads, int64_t seq_len);
int nsa_dense_decode(const void* q, const void* k, const void* v, void* o,
                     int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                     int64_t cache_len, int64_t seq_len, float sm_scale,
                     void* workspace, size_t workspace_bytes, nsa_stream_t stream);

/* ------------------------------------------------------------------ sparse
 * StreamingLLM sink + sliding-window decode over a [B, Hkv, sink+window, D]
 * cache.  Replaces sparse_kernel.py:105-118 sparse_decode_attention(q,
 * k_cache, v_cache, seq_len, window, sink, sm_scale) and its kernel
 * sparse_kernel.py:67-102 with the slot rule of _kv_indices
 * (sparse_kernel.py:15-46):
 *   sink slot s < sink valid iff s < seq_len;
 *   window slot s holds logical window index i = (s - sink - head) mod window,
 *   position seq_len - window + i, valid iff that position >= sink.
 * head = 0 is the reference's compacted layout; head = (seq_len - sink) mod
 * window is a ring buffer written at slot sink + (pos - sink) mod window.
 * seq_lens (int64 [B], device) and ring_heads (int32 [B], device) are
 * optional per-sequence overrides; pass NULL to use seq_len / head 0. */
size_t nsa_sparse_workspace_bytes(int64_t batch, int64_t n_kv_heads, int64_t window, int64_t sink);
int nsa_sparse_decode(const void* q, const void* k_cache, const void* v_cache, void* o,
                      int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                      int64_t window, int64_t sink, int64_t seq_len,
                      const int64_t* seq_lens, const int32_t* ring_heads, float sm_scale,
                      void* workspace, size_t workspace_bytes, nsa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NSA_B200_H_ */
