// Prefix-KV attention for one denoising step (at most 128 / rep forwarded positions), tcgen05.
//
// Semantics are those of attn_prefix_kernel (attention.cuh): the reference SDPA with the d2f
// block-causal mask (python/src/edllm/backends/mlx_ops.py:191-288, 347-443), GQA with the rep
// query heads of one KV head packed with the positions into the M = 128 rows of the UMMA
// (row r = position r / rep, head g * rep + r % rep).
//
// Work split, per KV head g: `splits` CTAs share the visible keys in balanced runs of 64-key
// sub-tiles, at most kDaMaxSub per CTA (one CTA per SM). A CTA
//   1. streams its K and V^T sub-tiles into shared memory with TMA. Sub-tiles that lie wholly
//      before the first forwarded position hold final K/V from earlier steps and are requested
//      before the programmatic-dependent-launch wait, so they stream while the QKV linear is
//      still running; the rest (and Q) are requested after it;
//   2. computes S_j = Q K_j^T for every sub-tile into TMEM (one 64-column block each);
//   3. runs a two-pass softmax over its keys with two threads per live row (pass 1: row max,
//      pass 2: exp2, the bf16 P written over the consumed K sub-tile), in the log2 domain;
//   4. accumulates O = sum_j P_j V_j on the tensor cores into TMEM;
//   5. with one split, normalises and writes bf16; otherwise writes its unnormalised f32 rows and
//      (m, l) to a partial buffer that attn_merge_kernel combines (rescale by exp2(m_i - max m),
//      sum in split order, normalise, write bf16).
// All waits are bounded (common.cuh); on a timeout the CTA records the error and unwinds.
#pragma once
#include "attention.cuh"

namespace drt {

constexpr int kDaMaxSub = 4;                    // 64-key sub-tiles per CTA
constexpr int kDaMaxSplits = 64;                // CTAs per KV head
constexpr int kDaQBytes = 2 * 128 * 128;        // Q: two 64-d atoms x 128 rows
constexpr int kDaKBytes = 2 * 64 * 128;         // K sub-tile: two 64-d atoms x 64 keys
constexpr int kDaVBytes = 128 * 128;            // V^T sub-tile: 128 d rows x 64 keys
constexpr int kDaSubBytes = kDaKBytes + kDaVBytes;
constexpr int kDaThreads = 256;
// Q | sub-tiles | row-statistics exchange | barriers
constexpr size_t kDaBodyBytes = kDaQBytes + static_cast<size_t>(kDaMaxSub) * kDaSubBytes;
constexpr size_t kDaRedFloats = 4 * 128;        // softmax row-statistics exchange
constexpr size_t kDaSmemBytes = 1024 + kDaBodyBytes + kDaRedFloats * 4 + 256;

struct DecAttnArgs {
  int nq, nkv, rep;
  int rows;               // query positions covered (<= 128 / rep)
  const int* rows_dev;    // device-side live position count
  int q_pos0;
  const int* q_pos0_dev;  // device-side first forwarded position
  int kv_len;
  const int* kv_len_dev;
  int prompt_len, block_size, bidirectional;
  int kv_plane0;          // first cache plane of this layer
  int splits;             // CTAs per KV head
  __nv_bfloat16* out;     // [rows][nq * 128]
  float* part_o;          // splits > 1: [nkv][splits][128 rows][128] unnormalised f32 rows
  float* part_ml;         // splits > 1: [nkv][splits][128 rows][2] (row max in log2 units, row sum)
  int* status;
  float scale_log2;       // log2(e) / sqrt(head_dim)
};

__device__ __forceinline__ int da_limit(const DecAttnArgs& a, int q_pos, int kv_len) {
  if (a.bidirectional) return kv_len;
  int lim;
  if (q_pos < a.prompt_len) lim = a.prompt_len;
  else lim = a.prompt_len + ((q_pos - a.prompt_len) / a.block_size + 1) * a.block_size;
  return min(lim, kv_len);
}

__global__ void __launch_bounds__(kDaThreads, 1)
    attn_decode_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK64,
                       const __grid_constant__ CUtensorMap tmV, const DecAttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sSub = smem + kDaQBytes;  // [kDaMaxSub][K | V^T]
  float* red = reinterpret_cast<float*>(smem + kDaBodyBytes);  // [4][128]: m halves, l halves
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + kDaRedFloats);
  uint64_t* barQ = bars;
  uint64_t* barKV = bars + 1;                 // [kDaMaxSub]
  uint64_t* barS = bars + 1 + kDaMaxSub;
  uint64_t* barO = barS + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(barS + 2);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int S = a.splits;
  const int split = blockIdx.x;
  const int g = blockIdx.y;
  const int plane = a.kv_plane0 + g;

  if (tid == 0) {
    mbar_init(barQ, 1);
    for (int j = 0; j < kDaMaxSub; ++j) mbar_init(&barKV[j], 1);
    mbar_init(barS, 1);
    mbar_init(barO, 1);
    flags[0] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK64);
    tma_prefetch_desc(&tmV);
  }
  // Device-side geometry: written by the plan kernel of this step, which completed before the
  // kernel preceding this one started, so it is safe to read before the dependency wait.
  const int kv_len = a.kv_len_dev != nullptr ? *a.kv_len_dev : a.kv_len;
  const int q_pos0 = a.q_pos0_dev != nullptr ? *a.q_pos0_dev : a.q_pos0;
  const int n_sub = (kv_len + 63) / 64;
  const int sub0 = static_cast<int>((static_cast<long long>(split) * n_sub) / S);
  const int sub1 = static_cast<int>((static_cast<long long>(split + 1) * n_sub) / S);
  const int nt = min(kDaMaxSub, max(0, sub1 - sub0));
  // Sub-tiles wholly before the first forwarded position hold final K/V.
  const int n_final = max(0, min(nt, q_pos0 / 64 - sub0));
  auto load_sub = [&](int j) {
    uint8_t* st = sSub + static_cast<size_t>(j) * kDaSubBytes;
    const int key0 = (sub0 + j) * 64;
    mbar_expect_tx(&barKV[j], kDaSubBytes);
    tma_load_3d(st, &tmK64, &barKV[j], 0, key0, plane);
    tma_load_3d(st + 64 * 128, &tmK64, &barKV[j], 64, key0, plane);
    tma_load_3d(st + kDaKBytes, &tmV, &barKV[j], key0, 0, plane);
  };
  if (tid == 0)
    for (int j = 0; j < n_final; ++j) load_sub(j);
  if (warp == 0) {
    tmem_alloc(tmem_slot, kDaMaxSub * 64 >= 128 ? kDaMaxSub * 64 : 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  griddep_wait();
  int rows_valid = a.rows;
  if (a.rows_dev != nullptr) rows_valid = min(rows_valid, *a.rows_dev);
  rows_valid = max(0, min(rows_valid, 128 / a.rep));
  const int rows_total = rows_valid * a.rep;
  if (tid == 0) {
    if (nt > 0) {
      const uint32_t qbytes = static_cast<uint32_t>(64 * 128 * 2);
      mbar_expect_tx(barQ, 2 * qbytes);
      tma_load_3d(sQ, &tmQ, barQ, 0, g * a.rep, 0);
      tma_load_3d(sQ + 128 * 128, &tmQ, barQ, 64, g * a.rep, 0);
      for (int j = n_final; j < nt; ++j) load_sub(j);
    }
  }
  griddep_launch_dependents();

  // ---- S_j = Q K_j^T (thread 0 issues; N = 64 keys per sub-tile)
  if (tid == 0) {
    bool ok = nt == 0 || mbar_wait(barQ, 0);
    const uint32_t idesc = idesc_bf16_f32(128, 64);
    for (int j = 0; j < nt && ok; ++j) {
      if (!mbar_wait(&barKV[j], 0)) { ok = false; break; }
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(sSub + static_cast<size_t>(j) * kDaSubBytes);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t qo = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
        const uint32_t ko = (kk >> 2) * (64 * 128) + (kk & 3) * 32;
        umma_bf16(tmem + j * 64, sdesc_kmajor_sw128(q_addr + qo), sdesc_kmajor_sw128(k_addr + ko), idesc, kk != 0 ? 1u : 0u);
      }
    }
    if (!ok) { record_error(a.status, DEV_TIMEOUT_TMA); flags[0] = 1; }
    umma_commit(barS);
  }
  const int r = tid & 127;
  const int half = tid >> 7;
  const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const int pos = r / a.rep;
  const bool row_ok = r < rows_total;
  const int lim = row_ok ? da_limit(a, q_pos0 + pos, kv_len) : 0;
  if (nt > 0 && !mbar_wait(barS, 0)) { record_error(a.status, DEV_TIMEOUT_MMA); flags[0] = 1; }
  tc_fence_after();

  // ---- pass 1: row max over this CTA's keys (thread covers 32 keys of every sub-tile)
  float mpart = -INFINITY;
  for (int j = 0; j < nt; ++j) {
    float sv[32];
    tmem_ld32(tmem + lane_off + j * 64 + half * 32, sv);
    const int k0 = (sub0 + j) * 64 + half * 32;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (k0 + i < lim) mpart = fmaxf(mpart, sv[i] * a.scale_log2);
  }
  red[half * 128 + r] = mpart;
  __syncthreads();
  const float m = fmaxf(red[r], red[128 + r]);
  // ---- pass 2: P = exp2(s - m) as bf16 over the consumed K sub-tile; partial row sums
  float lpart = 0.0f;
  for (int j = 0; j < nt; ++j) {
    float sv[32];
    tmem_ld32(tmem + lane_off + j * 64 + half * 32, sv);
    const int k0 = (sub0 + j) * 64 + half * 32;
    uint8_t* sP = sSub + static_cast<size_t>(j) * kDaSubBytes;  // [128 rows][64 keys] SW128
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      __align__(16) __nv_bfloat16 t[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int i = c * 8 + e;
        const float p = (k0 + i < lim) ? exp2f(sv[i] * a.scale_log2 - m) : 0.0f;
        t[e] = __float2bfloat16_rn(p);
        lpart += __bfloat162float(t[e]);
      }
      const int chunk = ((half * 32 + c * 8) >> 3) ^ (r & 7);
      *reinterpret_cast<uint4*>(sP + r * 128 + chunk * 16) = *reinterpret_cast<const uint4*>(t);
    }
  }
  red[256 + half * 128 + r] = lpart;
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  const float l = red[256 + r] + red[384 + r];

  // ---- O = sum_j P_j V_j into TMEM columns [0, 128) (the S columns are consumed)
  if (tid == 0) {
    tc_fence_after();
    const uint32_t idesc = idesc_bf16_f32(128, 128);
    for (int j = 0; j < nt; ++j) {
      const uint32_t p_addr = smem_u32(sSub + static_cast<size_t>(j) * kDaSubBytes);
      const uint32_t v_addr = p_addr + kDaKBytes;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16(tmem, sdesc_kmajor_sw128(p_addr + kk * 32), sdesc_kmajor_sw128(v_addr + kk * 32), idesc, (j | kk) != 0 ? 1u : 0u);
    }
    umma_commit(barO);
  }
  if (nt > 0 && !mbar_wait(barO, 0)) { record_error(a.status, DEV_TIMEOUT_MMA); flags[0] = 1; }
  tc_fence_after();
  float o[64];
  if (nt > 0) {
    tmem_ld32(tmem + lane_off + half * 64, o);
    tmem_ld32(tmem + lane_off + half * 64 + 32, o + 32);
  } else {
#pragma unroll
    for (int d = 0; d < 64; ++d) o[d] = 0.0f;
  }
  const float m_out = nt > 0 ? m : -INFINITY;
  const float l_out = nt > 0 ? l : 0.0f;

  if (row_ok && flags[0] == 0) {
    if (S == 1) {
      const float inv = l_out > 0.0f ? 1.0f / l_out : 0.0f;
      const int head = g * a.rep + (r - pos * a.rep);
      __nv_bfloat16* dst = a.out + (static_cast<size_t>(pos) * a.nq + head) * 128 + half * 64;
#pragma unroll
      for (int d = 0; d < 64; d += 8) {
        __align__(16) __nv_bfloat16 t[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) t[e] = __float2bfloat16_rn(o[d + e] * inv);
        *reinterpret_cast<uint4*>(dst + d) = *reinterpret_cast<const uint4*>(t);
      }
    } else {
      const size_t prow = (static_cast<size_t>(g) * S + split) * 128 + r;
      float* dst = a.part_o + prow * 128 + half * 64;
#pragma unroll
      for (int d = 0; d < 64; d += 4) *reinterpret_cast<float4*>(dst + d) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
      if (half == 0) *reinterpret_cast<float2*>(a.part_ml + prow * 2) = make_float2(m_out, l_out);
    }
  }
  if (flags[0] != 0 && tid == 0) {
    if (nt > 0) mbar_wait(barQ, 0);
    for (int j = 0; j < nt; ++j) mbar_wait(&barKV[j], 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kDaMaxSub * 64 >= 128 ? kDaMaxSub * 64 : 128);
}

// Combine the split partials of attn_decode_kernel. One CTA per KV head and group of
// kDaMergeRows live rows; thread (row i, column d). Threads d < splits fetch split d's (m, l) into
// shared memory while every thread fetches its column of all splits, so the merge costs one
// round trip.
constexpr int kDaMergeRows = 4;
__global__ void __launch_bounds__(128 * kDaMergeRows)
    attn_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int splits, int rep, int nq,
                      int rows, const int* rows_dev, __nv_bfloat16* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  int rows_valid = rows;
  if (rows_dev != nullptr) rows_valid = min(rows_valid, *rows_dev);
  const int g = blockIdx.x;
  const int i = threadIdx.x >> 7;
  const int d = threadIdx.x & 127;
  const int r = blockIdx.y * kDaMergeRows + i;
  if (blockIdx.y * kDaMergeRows >= rows_valid * rep) return;
  const bool live = r < rows_valid * rep;
  __shared__ float sm[kDaMergeRows][kDaMaxSplits], sl[kDaMergeRows][kDaMaxSplits];
  const size_t base = static_cast<size_t>(g) * splits * 128 + r;  // row index of split 0
  if (live && d < splits) {
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(part_ml + (base + static_cast<size_t>(d) * 128) * 2));
    sm[i][d] = ml.x;
    sl[i][d] = ml.y;
  }
  float o[kDaMaxSplits];
#pragma unroll
  for (int sp = 0; sp < kDaMaxSplits; ++sp)
    o[sp] = (live && sp < splits) ? __ldcg(part_o + (base + static_cast<size_t>(sp) * 128) * 128 + d) : 0.0f;
  __syncthreads();
  if (!live) return;
  float mx = -INFINITY;
  for (int sp = 0; sp < splits; ++sp)
    if (sl[i][sp] > 0.0f) mx = fmaxf(mx, sm[i][sp]);
  float L = 0.0f, acc = 0.0f;
#pragma unroll
  for (int sp = 0; sp < kDaMaxSplits; ++sp) {
    if (sp < splits) {
      const float w = sl[i][sp] > 0.0f ? exp2f(sm[i][sp] - mx) : 0.0f;
      L += sl[i][sp] * w;
      acc += o[sp] * w;
    }
  }
  const int pos = r / rep;
  const int head = g * rep + (r - pos * rep);
  out[(static_cast<size_t>(pos) * nq + head) * 128 + d] = __float2bfloat16_rn(L > 0.0f ? acc / L : 0.0f);
}

}  // namespace drt
