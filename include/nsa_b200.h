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
 * module constants), so any batch size and any Hkv are accepted.  An empty
 * batch (B = 0) launches nothing and returns NSA_OK; its tensor pointers may
 * then be NULL (what zero-size tensors carry).
 *
 * Reproducibility: the sink+window and KIVI attention kernels let their warps
 * claim a unit's work as they free up, so the order in which partial sums are
 * accumulated -- and with it the last fp16 rounding of an output -- can differ
 * between launches on the same inputs.  Cache contents written by the append
 * and quantization paths are bit-exact; the dense path is deterministic.
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
/* Self-test of the failure path: one CTA waits, limit_ns at most, on a
 * barrier phase that nothing completes; the wait gives up and records
 * NSA_ERR_TIMEOUT for nsa_device_error, and the context stays usable. */
int nsa_selftest_wait_timeout(int64_t limit_ns, nsa_stream_t stream);
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


/* fp16 ring cache with per-unit lengths (no reference counterpart: the
 * reference builds the compacted cache on the host,
 * test_sparse_correctness.py:51-72).  Unit u = (b, kv_head) holds
 * unit_lens[u] (int64 [B*Hkv], device) tokens: position p < sink at slot p,
 * position p >= sink at slot sink + (p - sink) % window (dropped when window
 * is 0), so its ring head is (len - sink) % window and the attended set is
 * nsa_sparse_decode's.  nsa_ring_append stores one token per unit (new_k,
 * new_v f16 [B, Hkv, D]) and advances unit_lens; nsa_ring_decode attends
 * (workspace: nsa_sparse_workspace_bytes); nsa_ring_decode_step does both,
 * in one launch when every unit has its own CTA (sink + window <= 384), else
 * as append + decode. */
int nsa_ring_append(void* k_cache, void* v_cache, int64_t* unit_lens, const void* new_k, const void* new_v,
                    int64_t batch, int64_t n_kv_heads, int64_t head_dim, int64_t window, int64_t sink,
                    nsa_stream_t stream);
int nsa_ring_decode(const void* q, const void* k_cache, const void* v_cache, void* o,
                    int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                    int64_t window, int64_t sink, const int64_t* unit_lens, float sm_scale,
                    void* workspace, size_t workspace_bytes, nsa_stream_t stream);
int nsa_ring_decode_step(const void* q, void* k_cache, void* v_cache, void* o,
                         int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                         int64_t window, int64_t sink, int64_t* unit_lens, const void* new_k,
                         const void* new_v, float sm_scale, void* workspace, size_t workspace_bytes,
                         nsa_stream_t stream);

/* Same computation as nsa_sparse_decode, but allocates nothing and takes no
 * workspace.  No counterpart in the reference: it exists for callers that
 * cannot call cudaMalloc (or any allocator) where they decode, e.g. a host
 * runtime that reserves all device memory through its own pool, or a plain C
 * caller without a device allocator.  The split-K scratch lives in a static
 * 4 MiB device array inside this library (held by every GPU that loads it
 * until exit).  Only launches that split a unit over several CTAs use it
 * (caches of more than 384 slots with fewer units than SMs, or long enough
 * for stream-K); those whose
 * scratch does not fit are rejected with NSA_ERR_UNSUPPORTED, while shapes
 * that keep every unit whole (one unit per CTA) have no size limit.  The
 * first call on a device that needs the array looks it up and clears it --
 * make that call before any stream capture.  An empty batch returns 0
 * without any CUDA call.  All calls on a device share the array: calls that
 * overlap on the GPU race on it. */
int nsa_sparse_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* o,
                              int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                              int64_t window, int64_t sink, int64_t seq_len,
                              const int64_t* seq_lens, const int32_t* ring_heads, float sm_scale,
                              nsa_stream_t stream);

/* ------------------------------------------------------------------ KIVI
 * 2-bit KIVI quantization: K per channel over groups of 32 tokens, V per
 * token over groups of 32 channels, asymmetric, fp16 scale and zero point,
 * 4 codes per byte.  dtype of the input: 0 = float32, 1 = float16.
 *
 * Replaces quant_kernel.py:106-126 quantize_k_cache(k, group_size, bits) and
 * its kernel quant_kernel.py:44-103: k [B, Hkv, T, D] (T % 32 == 0) ->
 * packed u8 [B, Hkv, T/4, D], scale and zero f16 [B, Hkv, T/32, D].
 * Bit-exact with the reference (IEEE float32 division, round-half-up via
 * floor(x + 0.5), fp16 round-to-nearest-even stores). */
int nsa_kivi_quantize_k(const void* k, int dtype, void* packed, void* scale, void* zero,
                        int64_t batch, int64_t n_kv_heads, int64_t seq_len, int64_t head_dim,
                        int64_t group_size, int64_t bits, nsa_stream_t stream);
/* Replaces quant_kernel.py:193-214 quantize_v_cache(v, group_size, bits) and
 * its kernel quant_kernel.py:129-190: v [B, Hkv, T, D] (D % 32 == 0) ->
 * packed u8 [B, Hkv, T, D/4], scale and zero f16 [B, Hkv, T, D/32]. */
int nsa_kivi_quantize_v(const void* v, int dtype, void* packed, void* scale, void* zero,
                        int64_t batch, int64_t n_kv_heads, int64_t seq_len, int64_t head_dim,
                        int64_t group_size, int64_t bits, nsa_stream_t stream);
/* Host-callable dequantization of tokens [tok_start, tok_start + n_tokens)
 * (positions clamped into [0, seq_len)) to float32 [B, Hkv, n_tokens, D]:
 * s * (code - z) with the fp16-stored s and z.  Replaces the Triton-only
 * helpers quant_kernel.py:219-266 _dequantize_k_tile and :269-311
 * _dequantize_v_tile that test_dequantize_tile_isolated.py:28-63 wraps. */
int nsa_kivi_dequant_k(const void* packed, const void* scale, const void* zero, void* out,
                       int64_t batch, int64_t n_kv_heads, int64_t seq_len, int64_t head_dim,
                       int64_t tok_start, int64_t n_tokens, nsa_stream_t stream);
int nsa_kivi_dequant_v(const void* packed, const void* scale, const void* zero, void* out,
                       int64_t batch, int64_t n_kv_heads, int64_t seq_len, int64_t head_dim,
                       int64_t tok_start, int64_t n_tokens, nsa_stream_t stream);

/* KIVI sink + window decode over the reference's 14-tensor layout, as built
 * by build_quantized_kv_cache (quant_kernel.py:584-622):
 *   k_res, v_res      f16 [B, Hkv, R, D]          the R newest window tokens
 *   k_sink_*          u8 [B, Hkv, 8, D] + f16 [B, Hkv, 1, D] x2   sink padded
 *   v_sink_*          u8 [B, Hkv, 32, D/4] + f16 [B, Hkv, 32, D/32] x2
 *   k_win_*           u8 [B, Hkv, (W-R)/4, D] + f16 [B, Hkv, (W-R)/32, D] x2
 *   v_win_*           u8 [B, Hkv, W-R, D/4] + f16 [B, Hkv, W-R, D/32] x2
 * Slot validity follows _kv_indices (sparse_kernel.py:15-46) over the
 * compacted order sink | window-old | residual.  Replaces
 * quant_kernel.py:551-581 sparse_decode_attention_quantized and its kernel
 * quant_kernel.py:436-548.  Requires window >= residual,
 * (window - residual) % 32 == 0, sink <= 32, group_size 32, bits 2. */
size_t nsa_kivi_workspace_bytes(int64_t batch, int64_t n_kv_heads, int64_t window, int64_t residual);
int nsa_kivi_decode(const void* q, const void* k_res, const void* v_res,
                    const void* k_sink_packed, const void* k_sink_scale, const void* k_sink_zero,
                    const void* v_sink_packed, const void* v_sink_scale, const void* v_sink_zero,
                    const void* k_win_packed, const void* k_win_scale, const void* k_win_zero,
                    const void* v_win_packed, const void* v_win_scale, const void* v_win_zero,
                    void* o, int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                    int64_t seq_len, int64_t window, int64_t sink, int64_t residual,
                    int64_t group_size, int64_t bits, float sm_scale,
                    void* workspace, size_t workspace_bytes, nsa_stream_t stream);

/* Streaming KIVI cache (no reference counterpart: the reference quantizes
 * once at setup, quant_kernel.py:7-8).  Token p < sink is a sink token; token
 * p >= sink has stream index i = p - sink.  Unflushed stream tokens live in
 * an fp16 residual ring of R + 32 slots (slot i % (R+32)); when R + 32 are
 * unflushed, the oldest 32 are quantized (quantize_k / quantize_v math) into
 * window group slot g % NG of a ring of NG = (W - R) / 32 groups (dropped
 * when NG == 0).  Attention covers exactly StreamingLLM's set: the first
 * min(len, sink) tokens and stream tokens with p >= len - W.  When
 * (len - sink - R) % 32 == 0 and len >= sink + W the state equals
 * build_quantized_kv_cache of the same window.  All pointers are device
 * memory; unit_lens holds the token count of every (batch, kv_head) unit.
 *
 * Memory format (chosen so that a batch of groups, or a run of residual
 * slots, is one contiguous copy into shared memory):
 *   groups: u8 [B, Hkv, 1 + NG, 3072], one record per quantized group,
 *     record 0 the sink group, record 1 + s window slot s; a record holds
 *     K codes u8 [8][D] at byte 0, K scale f16 [D] at 1024, K zero f16 [D]
 *     at 1280, V codes u8 [32][D/4] at 1536, V scale f16 [32][D/32] at 2560,
 *     V zero f16 [32][D/32] at 2816 -- the group's share of the reference's
 *     k_/v_{sink,win}_{packed,scale,zero} tensors.
 *   k_res, v_res: f16 [B, Hkv, R + 32, D]; slot r stores logical 16-byte
 *     chunk c (channels 8c .. 8c+7) at chunk (c & 8) | ((c & 7) ^ (r & 7)). */
typedef struct {
  int64_t batch, n_kv_heads, head_dim;  /* head_dim must be 128 */
  int64_t window, sink, residual;       /* W; S in [1, 32]; R a positive multiple of 32 */
  int64_t n_groups;                     /* (W - R) / 32 if W >= R, else 0 */
  int64_t* unit_lens;                   /* [B * Hkv] tokens appended so far */
  void* sink_k;                         /* f16 [B, Hkv, S, D] unquantized sink tokens */
  void* sink_v;
  void* groups;                         /* u8 [B, Hkv, 1 + NG, 3072] group records */
  void* k_res, *v_res;                  /* f16 [B, Hkv, R + 32, D], chunk-permuted slots */
} nsa_kivi_stream_cache;

/* Append one token per (batch, kv_head): new_k, new_v f16 [B, Hkv, D];
 * quantizes a group when one completes and advances unit_lens. */
int nsa_kivi_append(const nsa_kivi_stream_cache* cache, const void* new_k, const void* new_v,
                    nsa_stream_t stream);
/* Decode q [B, 8*Hkv, D] against the streaming cache -> o. */
size_t nsa_kivi_stream_workspace_bytes(const nsa_kivi_stream_cache* cache);
/* Kernel launches one nsa_kivi_stream_decode_step of this cache takes on the
 * current device: 1 (append inside the decode launch) or 2 (append, then
 * decode); 0 for an invalid descriptor.  Computes the plan only. */
int nsa_kivi_stream_step_launches(const nsa_kivi_stream_cache* cache);
int nsa_kivi_stream_decode(const nsa_kivi_stream_cache* cache, const void* q, void* o, float sm_scale,
                           void* workspace, size_t workspace_bytes, nsa_stream_t stream);
/* One decode step: nsa_kivi_append(new_k, new_v) then nsa_kivi_stream_decode(q),
 * with the same results and cache state.  When every unit is decoded by a
 * single CTA (more units than half the CTA slots, or any number when a unit's
 * groups and residual all fit the kernel's stages, as at W <= 416 with
 * residual 128) both run in one launch: the
 * decode's CTA of each unit stores the token, quantizes a completed group or
 * the sink group itself, and attends over its staged copies.  Same workspace
 * as nsa_kivi_stream_decode.  No reference counterpart (the reference has no
 * append path). */
int nsa_kivi_stream_decode_step(const nsa_kivi_stream_cache* cache, const void* new_k, const void* new_v,
                                const void* q, void* o, float sm_scale, void* workspace, size_t workspace_bytes,
                                nsa_stream_t stream);
/* nsa_kivi_stream_decode_step for n_layers caches of one geometry (caches:
 * host array of n_layers descriptors; new_k, new_v, q, o: host arrays of
 * n_layers device pointers), results as n_layers separate calls.  When the
 * step runs in one launch per layer, up to 64 layers share one launch
 * (layer-major CTAs): the launch's fixed costs are paid once.  For decode
 * loops that have every layer's query at once.  The workspace is the
 * single-layer one.  No reference counterpart. */
int nsa_kivi_stream_decode_step_layers(const nsa_kivi_stream_cache* caches, int64_t n_layers,
                                       const void* const* new_k, const void* const* new_v, const void* const* q,
                                       void* const* o, float sm_scale, void* workspace, size_t workspace_bytes,
                                       nsa_stream_t stream);

/* ------------------------------------------------------------ host buffers
 * Decode entry points over HOST buffers, for callers whose queries and
 * outputs live in host memory (the reference's Python functions accept CPU
 * tensors the caller moves).  A pipe owns `depth` device staging slots (one
 * input + one output region each) and two copy streams: every call copies
 * its input in on the pipe's input stream, runs the decode on `stream` and
 * copies the output back on the pipe's output stream, ordered by events, so
 * consecutive calls overlap their copies with each other's decode.  A slot
 * is reused only after its previous decode and output copy have finished.
 * Host buffers should be pinned for the copies to be asynchronous.
 * nsa_host_pipe_begin orders the pipe's copies after `stream`'s prior work;
 * nsa_host_pipe_end orders `stream`'s later work after every output copy
 * (the outputs are in host memory once that point of `stream` is reached).
 * A pipe belongs to the device current at its creation.  No reference
 * counterpart. */
#define NSA_HOST_PIPE_MAX_DEPTH 8
typedef struct nsa_host_pipe nsa_host_pipe;
nsa_host_pipe* nsa_host_pipe_create(size_t in_bytes, size_t out_bytes, int depth); /* NULL on failure */
void nsa_host_pipe_destroy(nsa_host_pipe* pipe);
int nsa_host_pipe_begin(nsa_host_pipe* pipe, nsa_stream_t stream);
int nsa_host_pipe_end(nsa_host_pipe* pipe, nsa_stream_t stream);
/* nsa_kivi_stream_decode_step with x_host = [q | new_k | new_v] packed
 * (f16, B*8*Hkv*D + 2*B*Hkv*D elements) and the output to o_host. */
int nsa_kivi_stream_decode_step_host(nsa_host_pipe* pipe, const nsa_kivi_stream_cache* cache, const void* x_host,
                                     void* o_host, float sm_scale, void* workspace, size_t workspace_bytes,
                                     nsa_stream_t stream);
/* nsa_sparse_decode / nsa_dense_decode with q and o in host memory (the
 * caches stay on the device). */
int nsa_sparse_decode_host(nsa_host_pipe* pipe, const void* q_host, const void* k_cache, const void* v_cache,
                           void* o_host, int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                           int64_t window, int64_t sink, int64_t seq_len, const int64_t* seq_lens,
                           const int32_t* ring_heads, float sm_scale, void* workspace, size_t workspace_bytes,
                           nsa_stream_t stream);
int nsa_dense_decode_host(nsa_host_pipe* pipe, const void* q_host, const void* k, const void* v, void* o_host,
                          int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t cache_len,
                          int64_t seq_len, float sm_scale, void* workspace, size_t workspace_bytes,
                          nsa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NSA_B200_H_ */
