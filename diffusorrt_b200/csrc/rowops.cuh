// Row-wise kernels of the decode step: embedding gather into the f32 residual stream,
// RMSNorm to the bf16 matmul input, and the seeded synthetic weight generator.
#pragma once
#include "common.cuh"

namespace drt {

// h[r, :] = f32(E[tokens[pos0 + r], :])   (python/src/edllm/backends/mlx_forward.py:1538-1557)
// With ss != null (blockDim.x == 128, H % 128 == 0) it also writes the per-row partial sums of
// squares over each group of 128 features, ss[r * (H / 128) + g], reduced in the same fixed order
// as the residual epilogue of the decode linears (warp tree, then the four warps in order).
__global__ void embed_rows_kernel(const int* __restrict__ tokens, int pos0, const int* pos0_dev, int rows,
                                  const int* rows_dev, const __nv_bfloat16* __restrict__ table, int H,
                                  float* __restrict__ h, int vocab, int* status, float* ss) {
  griddep_wait();
  griddep_launch_dependents();
  int rows_valid = rows;
  if (rows_dev != nullptr) rows_valid = min(rows_valid, *rows_dev);
  const int r = blockIdx.x;
  if (r >= rows_valid) return;
  const int p0 = pos0_dev != nullptr ? *pos0_dev : pos0;
  const int tok = tokens[p0 + r];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) record_error(status, DEV_BAD_SHAPE);
    return;
  }
  const __nv_bfloat16* src = table + static_cast<size_t>(tok) * H;
  float* dst = h + static_cast<size_t>(r) * H;
  if (ss == nullptr) {
    for (int k = threadIdx.x * 2; k < H; k += blockDim.x * 2) {
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(src + k);
      *reinterpret_cast<float2*>(dst + k) = make_float2(__low2float(v), __high2float(v));
    }
    return;
  }
  __shared__ float part[4];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  for (int g = 0; g < H / 128; ++g) {
    const float x = __bfloat162float(src[g * 128 + t]);
    dst[g * 128 + t] = x;
    float q = __fmul_rn(x, x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    if (lane == 0) part[warp] = q;
    __syncthreads();
    if (t == 0) ss[static_cast<size_t>(r) * (H / 128) + g] = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
    __syncthreads();
  }
}

// out[r, :] = bf16((x * (1 / sqrt(mean(x^2) + eps))) * w) with x = h[src_row(r), :] in f32.
// The reference rms_norm (mlx_ops.py:21-35) keeps the f32 residual dtype and multiplies the
// weight in f32; the bf16 cast is the one the following linear applies (mlx_ops.py:122-125).
// src_row(r) = row_index[r] when row_index is given (the frontier gather before lm_head).
// Every thread issues all of its loads (up to kNormVec float4 of x and of w) before the first use,
// so a row costs one memory round trip. Requires H % 4 == 0 and H <= 4 * kNormVec * blockDim.x.
constexpr int kNormVec = 4;
__global__ void rmsnorm_bf16_kernel(const float* __restrict__ h, int ld_h, const int* row_index, int rows,
                                    const int* rows_dev, const float* __restrict__ w, float eps, int H,
                                    __nv_bfloat16* __restrict__ out, int ld_out) {
  griddep_wait();
  griddep_launch_dependents();
  int rows_valid = rows;
  if (rows_dev != nullptr) rows_valid = min(rows_valid, *rows_dev);
  const int r = blockIdx.x;
  if (r >= rows_valid) return;
  const int src = row_index != nullptr ? row_index[r] : r;
  const float4* x4 = reinterpret_cast<const float4*>(h + static_cast<size_t>(src) * ld_h);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const int nv = H >> 2;
  float4 xv[kNormVec], wv[kNormVec];
#pragma unroll
  for (int i = 0; i < kNormVec; ++i) {
    const int k = threadIdx.x + i * blockDim.x;
    if (k < nv) {
      xv[i] = __ldcg(x4 + k);
      wv[i] = __ldg(w4 + k);
    } else {
      xv[i] = wv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormVec; ++i) {
    ss = __fmaf_rn(xv[i].x, xv[i].x, ss);
    ss = __fmaf_rn(xv[i].y, xv[i].y, ss);
    ss = __fmaf_rn(xv[i].z, xv[i].z, ss);
    ss = __fmaf_rn(xv[i].w, xv[i].w, ss);
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float var = __fdiv_rn(red[0], static_cast<float>(H));
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  __nv_bfloat16* y = out + static_cast<size_t>(r) * ld_out;
#pragma unroll
  for (int i = 0; i < kNormVec; ++i) {
    const int k = threadIdx.x + i * blockDim.x;
    if (k < nv) {
      __align__(8) __nv_bfloat16 t[4];
      t[0] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(xv[i].x, scale), wv[i].x));
      t[1] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(xv[i].y, scale), wv[i].y));
      t[2] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(xv[i].z, scale), wv[i].z));
      t[3] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(xv[i].w, scale), wv[i].w));
      *reinterpret_cast<uint2*>(y + 4 * k) = *reinterpret_cast<const uint2*>(t);
    }
  }
}

// ---------------------------------------------------------------- synthetic weights
// A seeded, counter-based generator whose every step is integer arithmetic plus one f32
// multiply, so a NumPy restatement reproduces each bf16 weight bit for bit:
//   z = splitmix64_finalize(seed * K1 + tensor_id * K2 + index)
//   u = byte0(z) + byte1(z) + byte2(z) + byte3(z) - 510          (Irwin-Hall of 4 bytes)
//   w = bf16_rn(f32(u) * f32(std / 147.80020))                    (unit variance of u is 147.8^2)
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float synth_value(uint64_t seed, uint32_t tensor_id, uint64_t index, float scale) {
  const uint64_t z = mix64(seed * 0x9E3779B97F4A7C15ull + static_cast<uint64_t>(tensor_id) * 0xD1B54A32D192ED03ull + index);
  const int u = static_cast<int>(z & 0xFF) + static_cast<int>((z >> 8) & 0xFF) + static_cast<int>((z >> 16) & 0xFF) +
                static_cast<int>((z >> 24) & 0xFF) - 510;
  return __fmul_rn(static_cast<float>(u), scale);
}

// Fill rows [0, rows) x cols of a block of tensor `tensor_id` into a packed destination: block
// element (r, c) is logical element (r0 + r, c0 + c) of the full [*, full_cols] tensor (a
// tensor-parallel shard; r0 = c0 = 0 and full_cols = cols for a whole tensor), and block row r lands
// at dst row (r / grp) * grp_stride + grp_off + r % grp.
__global__ void synth_fill_kernel(__nv_bfloat16* dst, int64_t rows, int64_t cols, uint64_t seed, uint32_t tensor_id,
                                  float scale, int64_t grp, int64_t grp_stride, int64_t grp_off, int64_t r0, int64_t c0,
                                  int64_t full_cols) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const int64_t dr = (r / grp) * grp_stride + grp_off + r % grp;
    const uint64_t li = static_cast<uint64_t>((r0 + r) * full_cols + c0 + c);
    dst[dr * cols + c] = __float2bfloat16_rn(synth_value(seed, tensor_id, li, scale));
  }
}

// Tensor parallel, peer-memory form (reduce-scatter then all-gather, both through NVLink stores).
// Feature tile t (128 features of H) belongs to rank t % world.
//
// Bounded wait (thread 0 of each CTA) until flags[r] >= tp_flag_value(epoch, tag) for every rank r. Once one
// wait has run out, later ones do not wait again: the request is failed already (status word).
__device__ __forceinline__ bool tp_wait_flags(const unsigned long long* flags, const unsigned long long* epoch, int tag,
                                              int world, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const unsigned long long e = tp_flag_value(*reinterpret_cast<const volatile unsigned long long*>(epoch), tag);
    bool good = *reinterpret_cast<volatile int*>(status) != DEV_TIMEOUT_PEER;
    const uint64_t t0 = globaltimer_ns();
    for (int r = 0; r < world && good; ++r) {
      while (ld_acquire_sys(flags + r) < e) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          good = false;
          break;
        }
      }
    }
    if (!good) record_error(status, DEV_TIMEOUT_PEER);
    ok = good ? 1 : 0;
  }
  __syncthreads();
  return ok != 0;
}

// Raise this rank's flag (tp_flag_value(epoch, tag)) on every rank once all CTAs of the grid have made their
// peer stores visible (the last CTA to arrive raises it and resets the counter).
__device__ __forceinline__ void tp_raise_flags(unsigned long long* const* flag_of_rank, int world, int* count,
                                               const unsigned long long* epoch, int tag) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int total = static_cast<int>(gridDim.x * gridDim.y * gridDim.z);
    if (atomicAdd(count, 1) + 1 == total) {
      __threadfence_system();
      const unsigned long long e = tp_flag_value(*reinterpret_cast<const volatile unsigned long long*>(epoch), tag);
      for (int r = 0; r < world; ++r) st_release_sys(flag_of_rank[r], e);
      *count = 0;
    }
  }
}

struct TpStep {
  float* h;                             // [rows][H] residual (f32)
  const float* recv;                    // this rank's receive buffer: [world][slot] f32 partials
  int64_t slot;                         // rows_cap * H
  __nv_bfloat16* ag_dst[8];             // per rank: that rank's all-gather buffer ([rows][H] bf16)
  const __nv_bfloat16* ag;              // this rank's all-gather buffer
  const unsigned long long* rs_flags;   // this rank's reduce-scatter flags [world]
  const unsigned long long* ag_flags;   // this rank's all-gather flags [world]
  unsigned long long* ag_flag_of_rank[8];  // this rank's all-gather flag on each rank
  int* count;
  const unsigned long long* epoch;
  int tag, world, rank, rows, H;
  int* status;
};

// Reduce-scatter half: for the feature tiles this rank owns, sum the ranks' partials in rank order,
// round to bf16 once (the linear's output rounding), add to the residual and store the rounded sum
// into every other rank's all-gather buffer; then raise this rank's all-gather flag everywhere.
__global__ void tp_rs_kernel(const TpStep a) {
  griddep_wait();
  const bool ok = tp_wait_flags(a.rs_flags, a.epoch, a.tag, a.world, a.status);
  griddep_launch_dependents();
  if (ok) {
    const int tiles = a.H / 128;
    const int own = (tiles - a.rank + a.world - 1) / a.world;   // tiles t = rank + k * world
    const int64_t per_row = static_cast<int64_t>(own) * 32;      // float4 groups per row
    const int64_t total = per_row * a.rows;
    for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < total;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t row = g / per_row;
      const int64_t rem = g - row * per_row;
      const int t = a.rank + static_cast<int>(rem / 32) * a.world;
      const int64_t off = row * a.H + t * 128 + (rem % 32) * 4;
      // L2 reads: the peers' stores land in this GPU's L2, not in this SM's L1
      float4 acc = __ldcg(reinterpret_cast<const float4*>(a.recv + off));
      for (int r = 1; r < a.world; ++r) {
        const float4 x = __ldcg(reinterpret_cast<const float4*>(a.recv + r * a.slot + off));
        acc.x = __fadd_rn(acc.x, x.x);
        acc.y = __fadd_rn(acc.y, x.y);
        acc.z = __fadd_rn(acc.z, x.z);
        acc.w = __fadd_rn(acc.w, x.w);
      }
      const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
      const __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
      float4 hv = *reinterpret_cast<float4*>(a.h + off);
      hv.x = __fadd_rn(hv.x, __low2float(lo));
      hv.y = __fadd_rn(hv.y, __high2float(lo));
      hv.z = __fadd_rn(hv.z, __low2float(hi));
      hv.w = __fadd_rn(hv.w, __high2float(hi));
      *reinterpret_cast<float4*>(a.h + off) = hv;
      uint2 packed;
      packed.x = *reinterpret_cast<const uint32_t*>(&lo);
      packed.y = *reinterpret_cast<const uint32_t*>(&hi);
      for (int r = 0; r < a.world; ++r)
        if (r != a.rank) *reinterpret_cast<uint2*>(a.ag_dst[r] + off) = packed;
    }
  }
  tp_raise_flags(a.ag_flag_of_rank, a.world, a.count, a.epoch, a.tag);
}

// Two-rank form: every rank has received every rank's whole partial; once all flags are up it sums
// them in rank order and adds bf16(sum) to its residual (one kernel, no second exchange).
__global__ void tp_reduce_all_kernel(const TpStep a) {
  griddep_wait();
  const bool ok = tp_wait_flags(a.rs_flags, a.epoch, a.tag, a.world, a.status);
  griddep_launch_dependents();
  if (!ok) return;
  const int64_t total = static_cast<int64_t>(a.rows) * a.H / 4;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 acc = __ldcg(reinterpret_cast<const float4*>(a.recv) + g);
    for (int r = 1; r < a.world; ++r) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(a.recv + r * a.slot) + g);
      acc.x = __fadd_rn(acc.x, x.x);
      acc.y = __fadd_rn(acc.y, x.y);
      acc.z = __fadd_rn(acc.z, x.z);
      acc.w = __fadd_rn(acc.w, x.w);
    }
    float4 hv = reinterpret_cast<float4*>(a.h)[g];
    hv.x = __fadd_rn(hv.x, __bfloat162float(__float2bfloat16_rn(acc.x)));
    hv.y = __fadd_rn(hv.y, __bfloat162float(__float2bfloat16_rn(acc.y)));
    hv.z = __fadd_rn(hv.z, __bfloat162float(__float2bfloat16_rn(acc.z)));
    hv.w = __fadd_rn(hv.w, __bfloat162float(__float2bfloat16_rn(acc.w)));
    reinterpret_cast<float4*>(a.h)[g] = hv;
  }
}

// All-gather half: add the other ranks' rounded sums for the feature tiles they own.
__global__ void tp_ag_kernel(const TpStep a) {
  griddep_wait();
  const bool ok = tp_wait_flags(a.ag_flags, a.epoch, a.tag, a.world, a.status);
  griddep_launch_dependents();
  if (!ok) return;
  const int64_t per_row = static_cast<int64_t>(a.H) / 4;
  const int64_t total = per_row * a.rows;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = g / per_row;
    const int f = static_cast<int>(g - row * per_row) * 4;
    if ((f >> 7) % a.world == a.rank) continue;
    const int64_t off = row * a.H + f;
    const uint2 packed = __ldcg(reinterpret_cast<const uint2*>(a.ag + off));
    const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&packed.x);
    const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&packed.y);
    float4 hv = *reinterpret_cast<float4*>(a.h + off);
    hv.x = __fadd_rn(hv.x, __low2float(lo));
    hv.y = __fadd_rn(hv.y, __high2float(lo));
    hv.z = __fadd_rn(hv.z, __low2float(hi));
    hv.w = __fadd_rn(hv.w, __high2float(hi));
    *reinterpret_cast<float4*>(a.h + off) = hv;
  }
}

// Holds the kernels after it until every rank's vocabulary-parallel lm_head has stored its logit
// tiles here (a.rs_flags: this rank's lm_head flag array, a.tag: the head's tag). Bounded.
__global__ void tp_gather_wait_kernel(const TpStep a) {
  griddep_wait();
  tp_wait_flags(a.rs_flags, a.epoch, a.tag, a.world, a.status);
  griddep_launch_dependents();
}

__global__ void tp_tick_kernel(unsigned long long* epoch) {
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) *epoch += 1ull;
}

// h[i] += bf16(part[i]) for i < n: the residual add after a tensor-parallel all-reduce of f32
// linear partials (the linear's bf16 output rounding applied to the reduced sum).
__global__ void resid_add_bf16r_kernel(float* __restrict__ h, const float* __restrict__ part, int64_t n) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 a = reinterpret_cast<float4*>(h)[i];
    const float4 b = reinterpret_cast<const float4*>(part)[i];
    a.x = __fadd_rn(a.x, __bfloat162float(__float2bfloat16_rn(b.x)));
    a.y = __fadd_rn(a.y, __bfloat162float(__float2bfloat16_rn(b.y)));
    a.z = __fadd_rn(a.z, __bfloat162float(__float2bfloat16_rn(b.z)));
    a.w = __fadd_rn(a.w, __bfloat162float(__float2bfloat16_rn(b.w)));
    reinterpret_cast<float4*>(h)[i] = a;
  }
  for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    h[i] = __fadd_rn(h[i], __bfloat162float(__float2bfloat16_rn(part[i])));
}

// Copy logical rows of a host-provided bf16 tensor (already on the device) into the packed
// destination with the same row map as synth_fill_kernel.
__global__ void pack_rows_kernel(__nv_bfloat16* dst, const __nv_bfloat16* src, int64_t rows, int64_t cols, int64_t grp,
                                 int64_t grp_stride, int64_t grp_off) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const int64_t dr = (r / grp) * grp_stride + grp_off + r % grp;
    dst[dr * cols + c] = src[i];
  }
}

__global__ void fill_f32_kernel(float* dst, int64_t n, float v) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = v;
}

__global__ void bf16_to_f32_kernel(float* dst, const __nv_bfloat16* src, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = __bfloat162float(src[i]);
}

}  // namespace drt
