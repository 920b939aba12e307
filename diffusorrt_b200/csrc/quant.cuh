// Group-wise 4-bit affine weight quantization (the linear-weight quantization the reference applies
// at load time, python/src/edllm/backends/mlx_dream.py:2090-2108 via mlx_ops.quantize_linear_weight,
// mlx_ops.py:63-94: per group of `group_size` consecutive inputs of one output row a scale and a
// bias in the weight dtype, w ~ scale * q + bias with q in [0, 2^bits - 1]).
//
// The reference delegates the rounding rules to mx.quantize, which is not part of the reference
// sources; this build defines them from that affine form, per group of 64 bf16 weights:
//   lo = min(w), hi = max(w)                                   (f32, exact)
//   scale = bf16((hi - lo) / 15), bias = bf16(lo)               (f32 IEEE divide, bf16 round-to-even)
//   q = clamp(rint((w - bias) / scale), 0, 15)   (f32 IEEE subtract and divide; q = 0 if scale = 0)
// Nibbles are packed two per byte, input 2j in the low nibble of byte j:
//   q_packed[row][j] = q[row][2j] | q[row][2j + 1] << 4;  scale / bias [row][group] bf16.
#pragma once
#include "common.cuh"

namespace drt {

__global__ void quantize_q4_kernel(const __nv_bfloat16* __restrict__ w, int64_t rows, int K, uint8_t* __restrict__ q,
                                   __nv_bfloat16* __restrict__ scale, __nv_bfloat16* __restrict__ bias) {
  const int groups = K / 64;
  const int64_t total = rows * groups;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / groups;
    const int g = static_cast<int>(idx - r * groups);
    const __nv_bfloat16* src = w + r * K + g * 64;
    float v[64];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + c * 8);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[c * 8 + e] = __bfloat162float(h[e]);
    }
    float lo = v[0], hi = v[0];
#pragma unroll
    for (int i = 1; i < 64; ++i) {
      lo = fminf(lo, v[i]);
      hi = fmaxf(hi, v[i]);
    }
    const __nv_bfloat16 sb = __float2bfloat16_rn(__fdiv_rn(__fsub_rn(hi, lo), 15.0f));
    const __nv_bfloat16 bb = __float2bfloat16_rn(lo);
    const float s = __bfloat162float(sb), b = __bfloat162float(bb);
    uint8_t* dst = q + r * (K / 2) + g * 32;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      int q0 = 0, q1 = 0;
      if (s > 0.0f) {
        q0 = static_cast<int>(rintf(__fdiv_rn(__fsub_rn(v[2 * j], b), s)));
        q1 = static_cast<int>(rintf(__fdiv_rn(__fsub_rn(v[2 * j + 1], b), s)));
        q0 = min(15, max(0, q0));
        q1 = min(15, max(0, q1));
      }
      dst[j] = static_cast<uint8_t>(q0 | (q1 << 4));
    }
    scale[r * groups + g] = sb;
    bias[r * groups + g] = bb;
  }
}

// Group-wise int8 weight-only quantization (the CUDA `int8_weight_only` precision the SDK names,
// python/src/edllm/backends/device_runtime.py:19-56: int8 weights, one scale per group of 64 inputs of
// a row, "weight-group-absmax" calibration; the reference's packing and rounding live in its private
// engine, so this build defines them), per group of 64 bf16 weights:
//   amax = max |w|                                              (f32, exact)
//   scale = bf16(amax / 127)                                    (f32 IEEE divide, bf16 round-to-even)
//   q = clamp(rint(w / scale), -127, 127)                       (f32 IEEE divide; q = 0 if scale = 0)
// stored as the unsigned byte q + 128 with bias = bf16(-128 * scale) (exact), so that the decode
// linear's affine dequantization scale * byte + bias gives scale * q exactly before its bf16 rounding:
//   q_packed[row][k] = q + 128;  scale / bias [row][group] bf16.
__global__ void quantize_q8_kernel(const __nv_bfloat16* __restrict__ w, int64_t rows, int K, uint8_t* __restrict__ q,
                                   __nv_bfloat16* __restrict__ scale, __nv_bfloat16* __restrict__ bias) {
  const int groups = K / 64;
  const int64_t total = rows * groups;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / groups;
    const int g = static_cast<int>(idx - r * groups);
    const __nv_bfloat16* src = w + r * K + g * 64;
    float v[64];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + c * 8);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[c * 8 + e] = __bfloat162float(h[e]);
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const __nv_bfloat16 sb = __float2bfloat16_rn(__fdiv_rn(amax, 127.0f));
    const float s = __bfloat162float(sb);
    uint8_t* dst = q + r * K + g * 64;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint32_t word = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int qi = 0;
        if (s > 0.0f) qi = min(127, max(-127, static_cast<int>(rintf(__fdiv_rn(v[c * 4 + e], s)))));
        word |= static_cast<uint32_t>(qi + 128) << (8 * e);
      }
      *reinterpret_cast<uint32_t*>(dst + c * 4) = word;
    }
    scale[r * groups + g] = sb;
    bias[r * groups + g] = __float2bfloat16_rn(-128.0f * s);
  }
}

}  // namespace drt
