// Decode entry points over host buffers: a pipe of device staging slots and
// two copy streams, so that the input copy of one call, the decode of
// another and the output copy of a third run at once (the copy engines and
// the SMs are separate resources).  Each call: input copy on the pipe's
// input stream -> decode on the caller's stream -> output copy on the pipe's
// output stream, ordered by events; slot b is reused only after its
// previous decode (input) and output copy have finished.
#include <cstdlib>
#include <new>

#include "host_util.h"

struct nsa_host_pipe {
  int device = -1;
  int depth = 0;
  size_t in_bytes = 0, out_bytes = 0, slot_bytes = 0;
  uint8_t* dev = nullptr;
  cudaStream_t s_in = nullptr, s_out = nullptr;
  cudaEvent_t ev_in[NSA_HOST_PIPE_MAX_DEPTH] = {}, ev_comp[NSA_HOST_PIPE_MAX_DEPTH] = {},
              ev_out[NSA_HOST_PIPE_MAX_DEPTH] = {};
  cudaEvent_t ev_mark = nullptr;
  uint64_t calls = 0;
};

namespace nsa {
namespace {

void destroy(nsa_host_pipe* p) {
  if (!p) return;
  int prev = -1;
  cudaGetDevice(&prev);
  if (p->device >= 0) cudaSetDevice(p->device);
  if (p->s_in) cudaStreamSynchronize(p->s_in);
  if (p->s_out) cudaStreamSynchronize(p->s_out);
  for (int i = 0; i < NSA_HOST_PIPE_MAX_DEPTH; ++i) {
    if (p->ev_in[i]) cudaEventDestroy(p->ev_in[i]);
    if (p->ev_comp[i]) cudaEventDestroy(p->ev_comp[i]);
    if (p->ev_out[i]) cudaEventDestroy(p->ev_out[i]);
  }
  if (p->ev_mark) cudaEventDestroy(p->ev_mark);
  if (p->s_in) cudaStreamDestroy(p->s_in);
  if (p->s_out) cudaStreamDestroy(p->s_out);
  if (p->dev) cudaFree(p->dev);
  if (prev >= 0) cudaSetDevice(prev);
  delete p;
}

int check_pipe(const nsa_host_pipe* p, size_t in_need, size_t out_need) {
  if (!p) return fail(NSA_ERR_INVALID, "null pipe");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != p->device)
    return fail(NSA_ERR_INVALID, "the pipe belongs to device %d, the current device is %d", p->device, dev);
  if (in_need > p->in_bytes || out_need > p->out_bytes)
    return fail(NSA_ERR_WORKSPACE, "pipe slots hold %zu / %zu bytes, the call needs %zu / %zu", p->in_bytes,
                p->out_bytes, in_need, out_need);
  return NSA_OK;
}

// One pipelined call: copy in_need bytes of x_host into the next slot, run
// `decode(x_dev, o_dev)` on `stream`, copy out_need bytes of the slot's
// output to o_host.
template <typename Decode>
int pipe_call(nsa_host_pipe* p, const void* x_host, size_t in_need, void* o_host, size_t out_need,
              cudaStream_t stream, Decode&& decode) {
  int rc = check_pipe(p, in_need, out_need);
  if (rc) return rc;
  if ((in_need > 0 && !x_host) || (out_need > 0 && !o_host)) return fail(NSA_ERR_INVALID, "null host buffer");
  const int b = static_cast<int>(p->calls % p->depth);
  const bool reuse = p->calls >= static_cast<uint64_t>(p->depth);
  uint8_t* x_dev = p->dev + b * p->slot_bytes;
  uint8_t* o_dev = x_dev + p->in_bytes;
  cudaError_t e = cudaSuccess;
  if (reuse) e = cudaStreamWaitEvent(p->s_in, p->ev_comp[b], 0);  // the slot's last decode has read its input
  if (e == cudaSuccess) e = cudaMemcpyAsync(x_dev, x_host, in_need, cudaMemcpyHostToDevice, p->s_in);
  if (e == cudaSuccess) e = cudaEventRecord(p->ev_in[b], p->s_in);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, p->ev_in[b], 0);
  if (e == cudaSuccess && reuse) e = cudaStreamWaitEvent(stream, p->ev_out[b], 0);  // its output was copied out
  if (e != cudaSuccess) return cuda_fail(e, "host pipe input");
  rc = decode(static_cast<const void*>(x_dev), static_cast<void*>(o_dev));
  if (rc) return rc;
  e = cudaEventRecord(p->ev_comp[b], stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_out, p->ev_comp[b], 0);
  if (e == cudaSuccess) e = cudaMemcpyAsync(o_host, o_dev, out_need, cudaMemcpyDeviceToHost, p->s_out);
  if (e == cudaSuccess) e = cudaEventRecord(p->ev_out[b], p->s_out);
  if (e != cudaSuccess) return cuda_fail(e, "host pipe output");
  ++p->calls;
  return NSA_OK;
}

}  // namespace
}  // namespace nsa

using namespace nsa;

extern "C" {

nsa_host_pipe* nsa_host_pipe_create(size_t in_bytes, size_t out_bytes, int depth) {
  clear_error();
  if (depth < 1 || depth > NSA_HOST_PIPE_MAX_DEPTH || in_bytes == 0 || out_bytes == 0) {
    fail(NSA_ERR_INVALID, "need 1 <= depth <= %d and non-zero slot sizes", NSA_HOST_PIPE_MAX_DEPTH);
    return nullptr;
  }
  nsa_host_pipe* p = new (std::nothrow) nsa_host_pipe();
  if (!p) {
    fail(NSA_ERR_INVALID, "out of host memory");
    return nullptr;
  }
  cudaError_t e = cudaGetDevice(&p->device);
  p->depth = depth;
  p->in_bytes = (in_bytes + 255) & ~size_t(255);
  p->out_bytes = (out_bytes + 255) & ~size_t(255);
  p->slot_bytes = p->in_bytes + p->out_bytes;
  if (e == cudaSuccess) e = cudaMalloc(&p->dev, p->slot_bytes * depth);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->s_in, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->s_out, cudaStreamNonBlocking);
  for (int i = 0; i < depth && e == cudaSuccess; ++i) {
    e = cudaEventCreateWithFlags(&p->ev_in[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->ev_comp[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->ev_out[i], cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->ev_mark, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    cuda_fail(e, "nsa_host_pipe_create");
    destroy(p);
    return nullptr;
  }
  return p;
}

void nsa_host_pipe_destroy(nsa_host_pipe* pipe) { destroy(pipe); }

int nsa_host_pipe_begin(nsa_host_pipe* pipe, nsa_stream_t stream) {
  clear_error();
  int rc = check_pipe(pipe, 0, 0);
  if (rc) return rc;
  cudaError_t e = cudaEventRecord(pipe->ev_mark, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pipe->s_in, pipe->ev_mark, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pipe->s_out, pipe->ev_mark, 0);
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "nsa_host_pipe_begin");
}

int nsa_host_pipe_end(nsa_host_pipe* pipe, nsa_stream_t stream) {
  clear_error();
  int rc = check_pipe(pipe, 0, 0);
  if (rc) return rc;
  cudaError_t e = cudaEventRecord(pipe->ev_mark, pipe->s_out);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, pipe->ev_mark, 0);
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "nsa_host_pipe_end");
}

int nsa_kivi_stream_decode_step_host(nsa_host_pipe* pipe, const nsa_kivi_stream_cache* cache, const void* x_host,
                                     void* o_host, float sm_scale, void* workspace, size_t workspace_bytes,
                                     nsa_stream_t stream) {
  clear_error();
  if (!cache) return fail(NSA_ERR_INVALID, "null cache");
  const size_t q_bytes = size_t(cache->batch) * cache->n_kv_heads * 8 * cache->head_dim * 2;
  const size_t kv_bytes = size_t(cache->batch) * cache->n_kv_heads * cache->head_dim * 2;
  return pipe_call(pipe, x_host, q_bytes + 2 * kv_bytes, o_host, q_bytes, stream,
                   [&](const void* x, void* o) {
                     const uint8_t* xb = static_cast<const uint8_t*>(x);
                     return nsa_kivi_stream_decode_step(cache, xb + q_bytes, xb + q_bytes + kv_bytes, xb, o, sm_scale,
                                                        workspace, workspace_bytes, stream);
                   });
}

int nsa_sparse_decode_host(nsa_host_pipe* pipe, const void* q_host, const void* k_cache, const void* v_cache,
                           void* o_host, int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                           int64_t window, int64_t sink, int64_t seq_len, const int64_t* seq_lens,
                           const int32_t* ring_heads, float sm_scale, void* workspace, size_t workspace_bytes,
                           nsa_stream_t stream) {
  clear_error();
  if (batch < 0 || n_heads < 0 || head_dim < 0) return fail(NSA_ERR_INVALID, "negative shape");
  const size_t q_bytes = size_t(batch) * n_heads * head_dim * 2;
  return pipe_call(pipe, q_host, q_bytes, o_host, q_bytes, stream, [&](const void* x, void* o) {
    return nsa_sparse_decode(x, k_cache, v_cache, o, batch, n_heads, n_kv_heads, head_dim, window, sink, seq_len,
                             seq_lens, ring_heads, sm_scale, workspace, workspace_bytes, stream);
  });
}

int nsa_dense_decode_host(nsa_host_pipe* pipe, const void* q_host, const void* k, const void* v, void* o_host,
                          int64_t batch, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t cache_len,
                          int64_t seq_len, float sm_scale, void* workspace, size_t workspace_bytes,
                          nsa_stream_t stream) {
  clear_error();
  if (batch < 0 || n_heads < 0 || head_dim < 0) return fail(NSA_ERR_INVALID, "negative shape");
  const size_t q_bytes = size_t(batch) * n_heads * head_dim * 2;
  return pipe_call(pipe, q_host, q_bytes, o_host, q_bytes, stream, [&](const void* x, void* o) {
    return nsa_dense_decode(x, k, v, o, batch, n_heads, n_kv_heads, head_dim, cache_len, seq_len, sm_scale,
                            workspace, workspace_bytes, stream);
  });
}

}  // extern "C"
