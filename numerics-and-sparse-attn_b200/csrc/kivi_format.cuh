// Memory format of the streaming KIVI cache (nsa_kivi_stream_cache in
// nsa_b200.h), shared by the append kernel (kivi_quant.cu) and the decode
// kernels (kivi_attn.cu).
//
// Quantized groups: one 3 KiB record per (unit, group), records of a unit
// contiguous, record 0 the sink group and record 1 + s window-group slot s.
// A record holds the six tensors the reference keeps apart (quant_kernel.py
// :44-214 layouts, one group's share of each), so that a run of groups is
// one contiguous copy:
//   [   0, 1024)  K codes   u8  [8][128]   byte i of channel c = tokens 4i..4i+3
//   [1024, 1280)  K scale   f16 [128]
//   [1280, 1536)  K zero    f16 [128]
//   [1536, 2560)  V codes   u8  [32][32]   byte j of token t = channels 4j..4j+3
//   [2560, 2816)  V scale   f16 [32][4]
//   [2816, 3072)  V zero    f16 [32][4]
//
// Residual ring: f16 [units][R + 32][128]; slot r keeps its 16-byte chunks
// (8 channels each) permuted within each 128-byte half: logical chunk c sits
// at (c & 8) | ((c & 7) ^ (r & 7)).  A contiguous copy of rows into shared
// memory is then bank-conflict free for 8-row matrix loads, which read one
// logical chunk of 8 consecutive slots.  The permutation is an involution.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace nsa {

constexpr int kRecBytes = 3072;
constexpr uint32_t kRecKP = 0, kRecKS = 1024, kRecKZ = 1280, kRecVP = 1536, kRecVS = 2560, kRecVZ = 2816;

struct GroupRec {
  uint8_t* kp;
  __half* ks;
  __half* kz;
  uint8_t* vp;
  __half* vs;
  __half* vz;
};

// Record `rec` (0: sink, 1 + s: window slot s) of `unit`.
__host__ __device__ __forceinline__ GroupRec group_rec(uint8_t* grp, int64_t unit, int n_groups, int rec) {
  uint8_t* b = grp + (unit * (n_groups + 1) + rec) * int64_t(kRecBytes);
  return GroupRec{b + kRecKP, reinterpret_cast<__half*>(b + kRecKS), reinterpret_cast<__half*>(b + kRecKZ),
                  b + kRecVP, reinterpret_cast<__half*>(b + kRecVS), reinterpret_cast<__half*>(b + kRecVZ)};
}

// Stored 16-byte chunk, within residual slot `slot`, of logical chunk ch.
__host__ __device__ __forceinline__ int res_chunk(int slot, int ch) { return (ch & 8) | ((ch & 7) ^ (slot & 7)); }

// Element index, within residual slot `slot`'s 128 elements, of channel c.
__host__ __device__ __forceinline__ int res_elem(int slot, int c) { return (res_chunk(slot, c >> 3) << 3) | (c & 7); }

}  // namespace nsa
