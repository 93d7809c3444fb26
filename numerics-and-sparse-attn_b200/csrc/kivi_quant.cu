// KIVI 2-bit quantization: setup-time quantizers (bit-exact with the
// reference quant_kernel.py:44-214), host-callable dequant of token ranges
// (the reference's _dequantize_k_tile / _dequantize_v_tile, quant_kernel.py
// :219-311, which it only exposes to Triton code), and the per-step
// quantize-on-append of the streaming cache (no reference counterpart).
//
// Arithmetic is IEEE float32 in the reference's order, written with explicit
// round-to-nearest intrinsics so no contraction or fast-math path can change
// a bit:  scale = (max - min) / 3, scale == 0 -> 1,
//         zero = floor(-min / scale + 0.5),
//         code = clamp(floor(x / scale + 0.5) + zero, 0, 3),
// scale and zero stored as float16 (round to nearest even; overflow -> inf),
// codes computed with the float32 scale.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kivi_format.cuh"
#include "quant_math.cuh"
#include "host_util.h"

namespace nsa {
namespace {

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p);
template <>
__device__ __forceinline__ float ld_f32<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_f32<__half>(const __half* p) { return __half2float(*p); }


// ---------------------------------------------------------------- K (per channel)
// One thread per (unit, 32-token group, channel).  in: [U, T, D]; packed
// [U, T/4, D] (byte i = tokens 4i..4i+3 at bits 0-1,2-3,4-5,6-7); scale/zero
// [U, T/32, D].
template <typename T>
__global__ void quantize_k_kernel(const T* __restrict__ in, uint8_t* __restrict__ packed,
                                  __half* __restrict__ scale, __half* __restrict__ zero, int64_t n_units,
                                  int64_t n_tok, int d) {
  const int64_t n_groups = n_tok / 32;
  const int64_t total = n_units * n_groups * d;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % d);
    const int64_t ug = idx / d;  // unit * n_groups + group
    const int64_t u = ug / n_groups, gi = ug % n_groups;
    const T* src = in + (u * n_tok + gi * 32) * d + c;
    float x[32];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      x[j] = ld_f32(src + int64_t(j) * d);
      mn = fminf(mn, x[j]);
      mx = fmaxf(mx, x[j]);
    }
    const GroupParams gp = group_params(mn, mx);
    scale[ug * d + c] = __float2half_rn(gp.scale);
    zero[ug * d + c] = __float2half_rn(gp.zero);
    uint8_t* dst = packed + (u * (n_tok / 4) + gi * 8) * d + c;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      uint32_t byte = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) byte |= code_of(x[4 * b + j], gp) << (2 * j);
      dst[int64_t(b) * d] = static_cast<uint8_t>(byte);
    }
  }
}

// ---------------------------------------------------------------- V (per token)
// One thread per (token, 32-channel group).  in: [U*T, D]; packed [U*T, D/4]
// (byte j = channels 4j..4j+3); scale/zero [U*T, D/32].
template <typename T>
__global__ void quantize_v_kernel(const T* __restrict__ in, uint8_t* __restrict__ packed,
                                  __half* __restrict__ scale, __half* __restrict__ zero, int64_t n_rows, int d) {
  const int ng = d / 32;
  const int64_t total = n_rows * ng;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row = idx / ng;
    const int q = static_cast<int>(idx % ng);
    const T* src = in + row * d + q * 32;
    float x[32];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      x[j] = ld_f32(src + j);
      mn = fminf(mn, x[j]);
      mx = fmaxf(mx, x[j]);
    }
    const GroupParams gp = group_params(mn, mx);
    scale[row * ng + q] = __float2half_rn(gp.scale);
    zero[row * ng + q] = __float2half_rn(gp.zero);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) lo |= code_of(x[j], gp) << (2 * j);
#pragma unroll
    for (int j = 0; j < 16; ++j) hi |= code_of(x[16 + j], gp) << (2 * j);
    // bytes in channel order: byte b holds channels 4b..4b+3 at bits 2*(c%4)
    uint8_t* dst = packed + row * (d / 4) + q * 8;
    *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
  }
}

// ---------------------------------------------------------------- dequant
// out[u, i, c] = s * (code - z) for tokens tok_start + i (clamped to
// [0, n_tok)), i < n_out.  K layout (tokens packed per byte).
__global__ void dequant_k_kernel(const uint8_t* __restrict__ packed, const __half* __restrict__ scale,
                                 const __half* __restrict__ zero, float* __restrict__ out, int64_t n_units,
                                 int64_t n_tok, int d, int64_t tok_start, int64_t n_out) {
  const int64_t total = n_units * n_out * d;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % d);
    const int64_t i = (idx / d) % n_out, u = idx / (d * n_out);
    int64_t t = tok_start + i;
    t = t < 0 ? 0 : (t >= n_tok ? n_tok - 1 : t);
    const uint32_t byte = packed[(u * (n_tok / 4) + t / 4) * d + c];
    const float code = static_cast<float>((byte >> (2 * (t % 4))) & 3u);
    const int64_t m = (u * (n_tok / 32) + t / 32) * d + c;
    out[idx] = __half2float(scale[m]) * (code - __half2float(zero[m]));
  }
}

// V layout (channels packed per byte).
__global__ void dequant_v_kernel(const uint8_t* __restrict__ packed, const __half* __restrict__ scale,
                                 const __half* __restrict__ zero, float* __restrict__ out, int64_t n_units,
                                 int64_t n_tok, int d, int64_t tok_start, int64_t n_out) {
  const int64_t total = n_units * n_out * d;
  for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % d);
    const int64_t i = (idx / d) % n_out, u = idx / (d * n_out);
    int64_t t = tok_start + i;
    t = t < 0 ? 0 : (t >= n_tok ? n_tok - 1 : t);
    const int64_t row = u * n_tok + t;
    const uint32_t byte = packed[row * (d / 4) + c / 4];
    const float code = static_cast<float>((byte >> (2 * (c % 4))) & 3u);
    const int64_t m = row * (d / 32) + c / 32;
    out[idx] = __half2float(scale[m]) * (code - __half2float(zero[m]));
  }
}

int grid_for(int64_t total, int threads) {
  const int sms = current_device().sm_count > 0 ? current_device().sm_count : 148;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = int64_t(sms) * 16;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

}  // namespace

// ---------------------------------------------------------------- append
// Quantize-on-append for the streaming cache (format in kivi_format.cuh).
// One CTA of 128 threads (thread = channel) per (batch, kv_head) unit; the
// unit's own length word orders everything, so no CTA depends on another.
__global__ void kivi_append_kernel(const __half* __restrict__ new_k, const __half* __restrict__ new_v,
                                   __half* __restrict__ sink_k16, __half* __restrict__ sink_v16,
                                   uint8_t* __restrict__ grp, __half* __restrict__ k_res, __half* __restrict__ v_res,
                                   int64_t* __restrict__ unit_lens, int sink, int residual, int n_groups) {
  constexpr int D = 128;
  grid_launch_dependents();
  grid_dependency_wait();  // the previous kernel may still read this cache
  const int64_t u = blockIdx.x;
  const int c = threadIdx.x;
  const int64_t pos = unit_lens[u];
  const int cap = residual + 32;
  const __half kx = new_k[u * D + c];
  const __half vx = new_v[u * D + c];
  __shared__ float vbuf[32][D + 1];  // V rows of a flushed group (float32, padded)
  GroupRec rec{};
  float x[32];  // K of channel c over the group's 32 tokens
  bool quantize = false;

  if (pos < sink) {
    // sink token: keep an fp16 copy, re-quantize the padded sink group (the n
    // real tokens, then copies of token 0)
    sink_k16[(u * sink + pos) * D + c] = kx;
    sink_v16[(u * sink + pos) * D + c] = vx;
    __syncthreads();
    const int n = static_cast<int>(pos) + 1;
    for (int j = 0; j < 32; ++j) {
      const int src = j < n ? j : 0;
      x[j] = __half2float(sink_k16[(u * sink + src) * D + c]);
      vbuf[j][c] = __half2float(sink_v16[(u * sink + src) * D + c]);
    }
    rec = group_rec(grp, u, n_groups, 0);
    quantize = true;
  } else {
    const int64_t i = pos - sink;  // stream index
    const int slot = static_cast<int>(i % cap);
    k_res[(u * cap + slot) * D + res_elem(slot, c)] = kx;
    v_res[(u * cap + slot) * D + res_elem(slot, c)] = vx;
    const int64_t f_old = (i - residual) >= 0 ? (i - residual) / 32 : 0;  // flushed before this token
    const int64_t f_new = (i + 1 - residual) >= 0 ? (i + 1 - residual) / 32 : 0;
    if (f_new > f_old && n_groups > 0) {
      // flush stream group f_old: indices [32 f_old, 32 f_old + 32) into window slot f_old % NG
      __syncthreads();
      const int64_t base = 32 * f_old;
      for (int j = 0; j < 32; ++j) {
        const int s = static_cast<int>((base + j) % cap);
        x[j] = __half2float(k_res[(u * cap + s) * D + res_elem(s, c)]);
        vbuf[j][c] = __half2float(v_res[(u * cap + s) * D + res_elem(s, c)]);
      }
      rec = group_rec(grp, u, n_groups, 1 + static_cast<int>(f_old % n_groups));
      quantize = true;
    }
  }
  if (quantize) {  // uniform across the CTA
    __syncthreads();
    // K: per channel over the 32 tokens
    float mn = INFINITY, mx = -INFINITY;
    for (int j = 0; j < 32; ++j) {
      mn = fminf(mn, x[j]);
      mx = fmaxf(mx, x[j]);
    }
    GroupParams gp = group_params(mn, mx);
    rec.ks[c] = __float2half_rn(gp.scale);
    rec.kz[c] = __float2half_rn(gp.zero);
    for (int bq = 0; bq < 8; ++bq) {
      uint32_t byte = 0;
      for (int j = 0; j < 4; ++j) byte |= code_of(x[4 * bq + j], gp) << (2 * j);
      rec.kp[bq * D + c] = static_cast<uint8_t>(byte);
    }
    // V: per token (32 tokens x 4 channel groups): thread = (token, group)
    const int tok = c >> 2, q = c & 3;
    float vmn = INFINITY, vmx = -INFINITY;
    for (int j = 0; j < 32; ++j) {
      vmn = fminf(vmn, vbuf[tok][q * 32 + j]);
      vmx = fmaxf(vmx, vbuf[tok][q * 32 + j]);
    }
    gp = group_params(vmn, vmx);
    rec.vs[tok * 4 + q] = __float2half_rn(gp.scale);
    rec.vz[tok * 4 + q] = __float2half_rn(gp.zero);
    uint32_t lo = 0, hi = 0;
    for (int j = 0; j < 16; ++j) lo |= code_of(vbuf[tok][q * 32 + j], gp) << (2 * j);
    for (int j = 0; j < 16; ++j) hi |= code_of(vbuf[tok][q * 32 + 16 + j], gp) << (2 * j);
    *reinterpret_cast<uint2*>(rec.vp + tok * 32 + q * 8) = make_uint2(lo, hi);
  }
  __syncthreads();  // every thread has read the length
  if (c == 0) unit_lens[u] = pos + 1;
}

}  // namespace nsa

using namespace nsa;

namespace {

int check_quant_args(const void* in, const void* p, const void* s, const void* z, int64_t n_units, int64_t n_tok,
                     int64_t d, int dtype) {
  if (n_units < 0 || n_tok < 0 || d <= 0) return fail(NSA_ERR_INVALID, "negative shape");
  // empty tensors may come with null pointers; there is nothing to do then
  if ((n_units == 0 || n_tok == 0) == false && (!in || !p || !s || !z))
    return fail(NSA_ERR_INVALID, "null tensor pointer");
  if (dtype != 0 && dtype != 1) return fail(NSA_ERR_UNSUPPORTED, "input dtype must be 0 (float32) or 1 (float16)");
  return NSA_OK;
}

}  // namespace

extern "C" {

int nsa_kivi_quantize_k(const void* k, int dtype, void* packed, void* scale, void* zero, int64_t batch,
                        int64_t n_kv_heads, int64_t seq_len, int64_t head_dim, int64_t group_size, int64_t bits,
                        nsa_stream_t stream) {
  clear_error();
  int rc = check_quant_args(k, packed, scale, zero, batch * n_kv_heads, seq_len, head_dim, dtype);
  if (rc) return rc;
  if (group_size != 32 || bits != 2) return fail(NSA_ERR_UNSUPPORTED, "only group_size=32, bits=2 are implemented");
  if (seq_len % 32) return fail(NSA_ERR_INVALID, "seq_len must be a multiple of group_size (got %lld)", (long long)seq_len);
  const int64_t units = batch * n_kv_heads;
  const int64_t total = units * (seq_len / 32) * head_dim;
  if (total == 0) return NSA_OK;
  const int th = 128;
  if (dtype == 0)
    quantize_k_kernel<float><<<grid_for(total, th), th, 0, stream>>>(
        static_cast<const float*>(k), static_cast<uint8_t*>(packed), static_cast<__half*>(scale),
        static_cast<__half*>(zero), units, seq_len, static_cast<int>(head_dim));
  else
    quantize_k_kernel<__half><<<grid_for(total, th), th, 0, stream>>>(
        static_cast<const __half*>(k), static_cast<uint8_t*>(packed), static_cast<__half*>(scale),
        static_cast<__half*>(zero), units, seq_len, static_cast<int>(head_dim));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "quantize_k launch");
}

int nsa_kivi_quantize_v(const void* v, int dtype, void* packed, void* scale, void* zero, int64_t batch,
                        int64_t n_kv_heads, int64_t seq_len, int64_t head_dim, int64_t group_size, int64_t bits,
                        nsa_stream_t stream) {
  clear_error();
  int rc = check_quant_args(v, packed, scale, zero, batch * n_kv_heads, seq_len, head_dim, dtype);
  if (rc) return rc;
  if (group_size != 32 || bits != 2) return fail(NSA_ERR_UNSUPPORTED, "only group_size=32, bits=2 are implemented");
  if (head_dim % 32) return fail(NSA_ERR_INVALID, "head_dim must be a multiple of group_size");
  const int64_t rows = batch * n_kv_heads * seq_len;
  if (rows > 0 && !aligned16(packed)) return fail(NSA_ERR_ALIGN, "packed must be 16-byte aligned");
  const int64_t total = rows * (head_dim / 32);
  if (total == 0) return NSA_OK;
  const int th = 128;
  if (dtype == 0)
    quantize_v_kernel<float><<<grid_for(total, th), th, 0, stream>>>(
        static_cast<const float*>(v), static_cast<uint8_t*>(packed), static_cast<__half*>(scale),
        static_cast<__half*>(zero), rows, static_cast<int>(head_dim));
  else
    quantize_v_kernel<__half><<<grid_for(total, th), th, 0, stream>>>(
        static_cast<const __half*>(v), static_cast<uint8_t*>(packed), static_cast<__half*>(scale),
        static_cast<__half*>(zero), rows, static_cast<int>(head_dim));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "quantize_v launch");
}

int nsa_kivi_dequant_k(const void* packed, const void* scale, const void* zero, void* out, int64_t batch,
                       int64_t n_kv_heads, int64_t seq_len, int64_t head_dim, int64_t tok_start, int64_t n_tokens,
                       nsa_stream_t stream) {
  clear_error();
  if (seq_len <= 0 || seq_len % 32 || n_tokens < 0 || head_dim <= 0)
    return fail(NSA_ERR_INVALID, "need seq_len > 0, seq_len % 32 == 0, n_tokens >= 0");
  const int64_t units = batch * n_kv_heads, total = units * n_tokens * head_dim;
  if (total == 0) return NSA_OK;
  if (!packed || !scale || !zero || !out) return fail(NSA_ERR_INVALID, "null tensor pointer");
  dequant_k_kernel<<<grid_for(total, 256), 256, 0, stream>>>(
      static_cast<const uint8_t*>(packed), static_cast<const __half*>(scale), static_cast<const __half*>(zero),
      static_cast<float*>(out), units, seq_len, static_cast<int>(head_dim), tok_start, n_tokens);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "dequant_k launch");
}

int nsa_kivi_dequant_v(const void* packed, const void* scale, const void* zero, void* out, int64_t batch,
                       int64_t n_kv_heads, int64_t seq_len, int64_t head_dim, int64_t tok_start, int64_t n_tokens,
                       nsa_stream_t stream) {
  clear_error();
  if (seq_len <= 0 || n_tokens < 0 || head_dim <= 0 || head_dim % 32)
    return fail(NSA_ERR_INVALID, "need seq_len > 0, n_tokens >= 0, head_dim % 32 == 0");
  const int64_t units = batch * n_kv_heads, total = units * n_tokens * head_dim;
  if (total == 0) return NSA_OK;
  if (!packed || !scale || !zero || !out) return fail(NSA_ERR_INVALID, "null tensor pointer");
  dequant_v_kernel<<<grid_for(total, 256), 256, 0, stream>>>(
      static_cast<const uint8_t*>(packed), static_cast<const __half*>(scale), static_cast<const __half*>(zero),
      static_cast<float*>(out), units, seq_len, static_cast<int>(head_dim), tok_start, n_tokens);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "dequant_v launch");
}

int nsa_kivi_append(const nsa_kivi_stream_cache* cache, const void* new_k, const void* new_v, nsa_stream_t stream) {
  clear_error();
  if (!cache) return fail(NSA_ERR_INVALID, "null cache");
  const nsa_kivi_stream_cache& c = *cache;
  int rc = kivi_check_stream_cache(c);
  if (rc) return rc;
  const int64_t units = c.batch * c.n_kv_heads;
  if (units == 0) return NSA_OK;
  if (!new_k || !new_v) return fail(NSA_ERR_INVALID, "null pointer");
  cudaError_t e = launch_kernel(
      kivi_append_kernel, dim3(static_cast<unsigned>(units)), dim3(128), 0, stream,
      static_cast<const __half*>(new_k), static_cast<const __half*>(new_v), static_cast<__half*>(c.sink_k),
      static_cast<__half*>(c.sink_v), static_cast<uint8_t*>(c.groups), static_cast<__half*>(c.k_res),
      static_cast<__half*>(c.v_res), c.unit_lens, static_cast<int>(c.sink), static_cast<int>(c.residual),
      static_cast<int>(c.n_groups));
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "kivi_append launch");
}

}  // extern "C"
