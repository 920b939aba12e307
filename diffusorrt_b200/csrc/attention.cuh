// Prefix-KV attention for block diffusion on the 5th-generation tensor cores.
//
// Semantics follow the reference SDPA (python/src/edllm/backends/mlx_ops.py:347-443) with the
// d2f_hybrid additive mask (mlx_ops.py:191-288, graph/numpyref.py:167-233): with
// eff(p) = -1 if p < prompt_len else (p - prompt_len) // block_size, query position q sees key
// position k iff eff(k) <= eff(q); "bidirectional" sees every key < kv_len. BD3 uses
// prompt_len = 0, so every 32-token block attends to itself and all earlier blocks.
//
// Work unit: one KV head g, one query tile and one slice of the keys. The query tile packs
// `rep` = nq/nkv query heads x P positions as the M = 128 rows of the UMMA (row r = position
// r / rep, head g*rep + r % rep), so GQA needs no K/V duplication. Per 128-key tile:
//   S = Q K^T       (tcgen05.mma, A = Q tile [128 x 128d], B = K tile [128 keys x 128d], TMEM)
//   P = softmax     (one thread per row: online max/sum in the log2 domain, P as bf16 in smem)
//   O_t = P V       (tcgen05.mma, A = P [128 x 128 keys], B = V^T tile [128d x 128 keys])
//   o = o * alpha + O_t in registers.
// K is cached as [nkv][pos][128] and V transposed as [nkv][128][pos], so both B operands are
// K-major 128-byte-swizzled TMA tiles. With splits > 1 the CTAs of one KV head form a thread-
// block cluster and merge their (o, m, l) partials through distributed shared memory in rank
// order.
#pragma once
#include "common.cuh"

namespace drt {

struct AttnArgs {
  int nq, nkv, rep;       // query heads, kv heads, nq / nkv
  int tile_pos;           // query positions per tile (P); rep * P <= 128
  int rows;               // query rows (positions) covered by the grid
  const int* rows_dev;    // optional device-side row count
  int q_pos0;             // absolute position of query row 0
  const int* q_pos0_dev;
  int kv_len;             // keys [0, kv_len) are valid
  const int* kv_len_dev;
  int prompt_len, block_size, bidirectional;
  int kv_plane0;          // first plane of this layer in the [L*nkv] cache planes
  int splits, tiles_per_split;  // splits = cluster size along z (1, 4, 8 or 16)
  __nv_bfloat16* out;     // [rows][nq*128]
  int* status;
  float scale_log2;       // log2(e) / sqrt(head_dim)
};

__device__ __forceinline__ int attn_limit(const AttnArgs& a, int q_pos, int kv_len) {
  if (a.bidirectional) return kv_len;
  int lim;
  if (q_pos < a.prompt_len) lim = a.prompt_len;
  else lim = a.prompt_len + ((q_pos - a.prompt_len) / a.block_size + 1) * a.block_size;
  return min(lim, kv_len);
}

constexpr int kAttnQBytes = 2 * 128 * 128;     // two 64-column atoms x 128 rows
constexpr int kAttnKBytes = 2 * 128 * 128;     // 128 keys x 128 d
constexpr int kAttnVBytes = 2 * 128 * 128;     // 128 d x 128 keys
constexpr int kAttnStageBytes = kAttnKBytes + kAttnVBytes;
constexpr int kAttnPBytes = 2 * 128 * 128;
constexpr int kAttnStages = 2;
constexpr int kAttnRowStride = 132;  // floats per received row (conflict-free float4 access)
constexpr size_t kAttnSmemBytes = 1024 + kAttnQBytes + kAttnStages * kAttnStageBytes + kAttnPBytes + 256;

// 2^x with the PTX approximate instruction (relative error within 2^-22 of the exact power; a
// subnormal result flushes to zero). P is rounded to bf16 right after, 2^-9 relative.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Columns [c, c + 64) of this thread's TMEM lane (two 32x32b.x32 loads), one wait for both, in the
// same statement so no use of the registers can be scheduled before the data lands.
__device__ __forceinline__ void tmem_ld32x2(uint32_t taddr, float* v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr), "r"(taddr + 32)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// Split-KV merge inside one cluster of S CTAs (one KV head). CTA r owns query rows
// [r*R, (r+1)*R), R = 128 / S. Every thread pushes its row's unnormalized (o, m, l) into the
// owner's receive buffer recv[src rank * R + row % R] with remote stores; after the cluster
// barrier the owner merges its rows over the S sources in rank order from local shared memory.
template <int S>
__device__ __forceinline__ void attn_push(const float* o_acc, float m_run, float l_run, float* recv, float* recv_ml,
                                          int tid) {
  constexpr int R = 128 / S;
  const uint32_t rank = cluster_ctarank();
  const uint32_t owner = static_cast<uint32_t>(tid / R);
  const int slot = static_cast<int>(rank) * R + (tid % R);
  const uint32_t dst = cluster_map(smem_u32(recv) + static_cast<uint32_t>(slot * kAttnRowStride * 4), owner);
#pragma unroll
  for (int d = 0; d < 128; d += 4)
    st_cluster_f32x4(dst + d * 4, make_float4(o_acc[d], o_acc[d + 1], o_acc[d + 2], o_acc[d + 3]));
  st_cluster_f32x2(cluster_map(smem_u32(recv_ml) + static_cast<uint32_t>(slot * 8), owner), m_run, l_run);
}

template <int S>
__device__ __forceinline__ void attn_merge(const AttnArgs& a, const float* recv, const float* recv_ml, int g, int row0,
                                           int rows_valid, int tid, bool failed) {
  constexpr int R = 128 / S;
  constexpr int ITEMS = R / 8;  // (row, 8-wide chunk) items per thread
  const uint32_t rank = cluster_ctarank();
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    const int item = it * 128 + tid;
    const int lr = item / 16;  // local row in [0, R)
    const int row = static_cast<int>(rank) * R + lr;
    const int d0 = (item % 16) * 8;
    float m_all = -INFINITY;
#pragma unroll
    for (int p = 0; p < S; ++p) m_all = fmaxf(m_all, recv_ml[(p * R + lr) * 2]);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float l_all = 0.0f;
#pragma unroll
    for (int p = 0; p < S; ++p) {
      const float m = recv_ml[(p * R + lr) * 2];
      const float l = recv_ml[(p * R + lr) * 2 + 1];
      const float w = (l == 0.0f || m == -INFINITY) ? 0.0f : exp2f(m - m_all);
      l_all += l * w;
      const float4 lo = *reinterpret_cast<const float4*>(recv + (p * R + lr) * kAttnRowStride + d0);
      const float4 hi = *reinterpret_cast<const float4*>(recv + (p * R + lr) * kAttnRowStride + d0 + 4);
      acc[0] += lo.x * w;
      acc[1] += lo.y * w;
      acc[2] += lo.z * w;
      acc[3] += lo.w * w;
      acc[4] += hi.x * w;
      acc[5] += hi.y * w;
      acc[6] += hi.z * w;
      acc[7] += hi.w * w;
    }
    const int r_pos = row / a.rep;
    const int r_q = row0 + r_pos;
    if (!failed && r_pos < a.tile_pos && r_q < rows_valid) {
      const int r_head = g * a.rep + (row - r_pos * a.rep);
      const float inv = l_all > 0.0f ? 1.0f / l_all : 0.0f;
      __align__(16) __nv_bfloat16 t[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) t[e] = __float2bfloat16_rn(acc[e] * inv);
      *reinterpret_cast<uint4*>(a.out + static_cast<size_t>(r_q) * a.nq * 128 + static_cast<size_t>(r_head) * 128 + d0) =
          *reinterpret_cast<const uint4*>(t);
    }
  }
}

__global__ void __launch_bounds__(128, 1)
    attn_prefix_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kAttnQBytes;
  uint8_t* sP = sKV + kAttnStages * kAttnStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kAttnPBytes);
  uint64_t* barQ = bars;
  uint64_t* fullKV = bars + 1;  // [kAttnStages]
  uint64_t* barS = bars + 1 + kAttnStages;
  uint64_t* barO = barS + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(barO + 1);
  int* sflag = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int qt = blockIdx.x;
  const int g = blockIdx.y;
  const int split = blockIdx.z;

  if (tid == 0) {
    mbar_init(barQ, 1);
    for (int s = 0; s < kAttnStages; ++s) mbar_init(&fullKV[s], 1);
    mbar_init(barS, 1);
    mbar_init(barO, 1);
    sflag[0] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem;
  const uint32_t tmem_o = tmem + 128;

  griddep_wait();
  griddep_launch_dependents();

  int rows_valid = a.rows;
  if (a.rows_dev != nullptr) rows_valid = min(rows_valid, *a.rows_dev);
  const int q_pos0 = a.q_pos0_dev != nullptr ? *a.q_pos0_dev : a.q_pos0;
  const int kv_len = a.kv_len_dev != nullptr ? *a.kv_len_dev : a.kv_len;
  const int row0 = qt * a.tile_pos;  // first query row of this tile

  // Key range of this CTA.
  const int last_row = min(row0 + a.tile_pos, rows_valid) - 1;
  const int kv_hi = last_row >= row0 ? attn_limit(a, q_pos0 + last_row, kv_len) : 0;
  const int n_kv_tiles = (kv_hi + 127) / 128;
  const int t_begin = split * a.tiles_per_split;
  const int t_end = min(n_kv_tiles, t_begin + a.tiles_per_split);
  const int ntiles = max(0, t_end - t_begin);

  // This thread's query row.
  const int r_local = tid / a.rep;
  const int h_local = tid - r_local * a.rep;
  const int q_row = row0 + r_local;
  const bool row_ok = (r_local < a.tile_pos) && (q_row < rows_valid);
  const int head = g * a.rep + h_local;
  const int lim = row_ok ? attn_limit(a, q_pos0 + q_row, kv_len) : 0;

  const int plane = a.kv_plane0 + g;
  if (tid == 0 && ntiles > 0) {
    const uint32_t qbytes = static_cast<uint32_t>(64 * a.rep * a.tile_pos * 2);
    mbar_expect_tx(barQ, 2 * qbytes);
    tma_load_3d(sQ, &tmQ, barQ, 0, g * a.rep, row0);
    tma_load_3d(sQ + 128 * 128, &tmQ, barQ, 64, g * a.rep, row0);
    for (int j = 0; j < min(kAttnStages, ntiles); ++j) {
      uint8_t* st = sKV + j * kAttnStageBytes;
      const int key0 = (t_begin + j) * 128;
      mbar_expect_tx(&fullKV[j], kAttnStageBytes);
      tma_load_3d(st, &tmK, &fullKV[j], 0, key0, plane);
      tma_load_3d(st + 128 * 128, &tmK, &fullKV[j], 64, key0, plane);
      tma_load_3d(st + kAttnKBytes, &tmV, &fullKV[j], key0, 0, plane);
      tma_load_3d(st + kAttnKBytes + 128 * 128, &tmV, &fullKV[j], key0 + 64, 0, plane);
    }
  }

  float o_acc[128];
#pragma unroll
  for (int d = 0; d < 128; ++d) o_acc[d] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;
  const uint32_t idesc = idesc_bf16_f32(128, 128);
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  bool failed = false;

  for (int j = 0; j < ntiles; ++j) {
    const int s = j % kAttnStages;
    uint8_t* st = sKV + s * kAttnStageBytes;
    const int key0 = (t_begin + j) * 128;
    if (tid == 0) {
      bool ok = (j > 0 || mbar_wait(barQ, 0)) && mbar_wait(&fullKV[s], (j / kAttnStages) & 1);
      if (!ok) {
        record_error(a.status, DEV_TIMEOUT_TMA);
        sflag[0] = 1;
      } else {
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ);
        const uint32_t k_addr = smem_u32(st);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          umma_bf16(tmem_s, sdesc_kmajor_sw128(q_addr + off), sdesc_kmajor_sw128(k_addr + off), idesc,
                    kk != 0 ? 1u : 0u);
        }
      }
      umma_commit(barS);
    }
    if (!mbar_wait(barS, j & 1)) { record_error(a.status, DEV_TIMEOUT_MMA); sflag[0] = 1; }
    tc_fence_after();
    __syncthreads();
    if (sflag[0]) { failed = true; break; }

    // Row softmax over this key tile: pass 1 max, pass 2 exponentials (TMEM re-read).
    float tile_max = -INFINITY;
#pragma unroll
    for (int cb = 0; cb < 128; cb += 32) {
      float sv[32];
      tmem_ld32(tmem_s + lane_off + cb, sv);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int kp = key0 + cb + i;
        const float x = (kp < lim) ? sv[i] * a.scale_log2 : -INFINITY;
        tile_max = fmaxf(tile_max, x);
      }
    }
    const float m_new = fmaxf(m_run, tile_max);
    const float alpha = (m_new == -INFINITY) ? 1.0f : exp2f(m_run - m_new);
    float psum = 0.0f;
#pragma unroll
    for (int cb = 0; cb < 128; cb += 32) {
      float sv[32];
      tmem_ld32(tmem_s + lane_off + cb, sv);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const int kp = key0 + cb + i;
        const float p0 = (kp < lim && m_new != -INFINITY) ? exp2f(sv[i] * a.scale_log2 - m_new) : 0.0f;
        const float p1 = (kp + 1 < lim && m_new != -INFINITY) ? exp2f(sv[i + 1] * a.scale_log2 - m_new) : 0.0f;
        const __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
        psum += __low2float(pb) + __high2float(pb);
        *reinterpret_cast<__nv_bfloat162*>(sP + sw128_offset(tid, cb + i, 128)) = pb;
      }
    }
    l_run = l_run * alpha + psum;
    m_run = m_new;
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    if (tid == 0) {
      tc_fence_after();
      const uint32_t p_addr = smem_u32(sP);
      const uint32_t v_addr = smem_u32(st + kAttnKBytes);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
        umma_bf16(tmem_o, sdesc_kmajor_sw128(p_addr + off), sdesc_kmajor_sw128(v_addr + off), idesc,
                  kk != 0 ? 1u : 0u);
      }
      umma_commit(barO);
    }
    if (!mbar_wait(barO, j & 1)) { record_error(a.status, DEV_TIMEOUT_MMA); sflag[0] = 1; }
    tc_fence_after();
    __syncwarp();
#pragma unroll
    for (int cb = 0; cb < 128; cb += 32) {
      float ov[32];
      tmem_ld32(tmem_o + lane_off + cb, ov);
#pragma unroll
      for (int i = 0; i < 32; ++i) o_acc[cb + i] = o_acc[cb + i] * alpha + ov[i];
    }
    // Stage s is free (its O MMA completed): refill it with tile j + kAttnStages.
    if (tid == 0 && j + kAttnStages < ntiles && !sflag[0]) {
      const int key1 = (t_begin + j + kAttnStages) * 128;
      mbar_expect_tx(&fullKV[s], kAttnStageBytes);
      tma_load_3d(st, &tmK, &fullKV[s], 0, key1, plane);
      tma_load_3d(st + 128 * 128, &tmK, &fullKV[s], 64, key1, plane);
      tma_load_3d(st + kAttnKBytes, &tmV, &fullKV[s], key1, 0, plane);
      tma_load_3d(st + kAttnKBytes + 128 * 128, &tmV, &fullKV[s], key1 + 64, 0, plane);
    }
    tc_fence_before();
    __syncthreads();
    if (sflag[0]) { failed = true; break; }
  }

  if (a.splits == 1) {
    if (!failed && row_ok) {
      const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      __nv_bfloat16* dst = a.out + static_cast<size_t>(q_row) * a.nq * 128 + static_cast<size_t>(head) * 128;
#pragma unroll
      for (int d = 0; d < 128; d += 8) {
        __align__(16) __nv_bfloat16 t[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) t[e] = __float2bfloat16_rn(o_acc[d + e] * inv);
        *reinterpret_cast<uint4*>(dst + d) = *reinterpret_cast<const uint4*>(t);
      }
    }
  } else {
    // Split-KV merge across the cluster (dims 1 x 1 x splits). The receive buffer overlays the
    // K/V stages, which peers may only write once this CTA's loads and UMMAs are done: arrive now,
    // wait before pushing.
    cluster_arrive();
    float* recv = reinterpret_cast<float*>(sKV);      // [128][kAttnRowStride]
    float* recv_ml = recv + 128 * kAttnRowStride;      // [128][2]
    const float mr = failed ? -INFINITY : m_run;
    const float lr = failed ? 0.0f : l_run;
    cluster_wait();
    switch (a.splits) {
      case 4: attn_push<4>(o_acc, mr, lr, recv, recv_ml, tid); break;
      case 8: attn_push<8>(o_acc, mr, lr, recv, recv_ml, tid); break;
      default: attn_push<16>(o_acc, mr, lr, recv, recv_ml, tid); break;
    }
    cluster_sync();
    switch (a.splits) {
      case 4: attn_merge<4>(a, recv, recv_ml, g, row0, rows_valid, tid, failed); break;
      case 8: attn_merge<8>(a, recv, recv_ml, g, row0, rows_valid, tid, failed); break;
      default: attn_merge<16>(a, recv, recv_ml, g, row0, rows_valid, tid, failed); break;
    }
  }
  if (failed && tid == 0) {
    mbar_wait(barQ, 0);
    for (int s = 0; s < min(kAttnStages, ntiles); ++s) mbar_wait(&fullKV[s], 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

}  // namespace drt

namespace drt {

// Attention over many query tiles (prompt prefill, full-canvas forward): the tiles and math of
// attn_prefix_kernel without split-KV, on 256 threads. The two threads of a query row (t and
// t + 128: same TMEM lanes, warps w and w + 4) split the row's 128 key columns for the softmax
// (row max and row sum exchanged through shared memory) and its 128 head dims for the output
// accumulator; and the S = Q K^T MMA of key tile j + 1 is issued into the second S buffer before
// the softmax of tile j, so the tensor cores work while the threads do.
constexpr int kAttnWThreads = 256;

__global__ void __launch_bounds__(kAttnWThreads, 1)
    attn_wide_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kAttnQBytes;
  uint8_t* sP = sKV + kAttnStages * kAttnStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kAttnPBytes);
  uint64_t* barQ = bars;
  uint64_t* fullKV = bars + 1;  // [kAttnStages]
  uint64_t* barS = bars + 1 + kAttnStages;  // [2]
  uint64_t* barO = barS + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(barO + 1);
  int* sflag = reinterpret_cast<int*>(tmem_slot + 1);
  __shared__ float red_m[kAttnWThreads];
  __shared__ float red_s[kAttnWThreads];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int half = warp >> 2;              // 0: key columns / dims 0..63, 1: 64..127
  const int r = (warp & 3) * 32 + lane;     // UMMA row = TMEM lane of this thread
  const int qt = blockIdx.x;
  const int g = blockIdx.y;

  if (tid == 0) {
    mbar_init(barQ, 1);
    for (int s = 0; s < kAttnStages; ++s) mbar_init(&fullKV[s], 1);
    mbar_init(&barS[0], 1);
    mbar_init(&barS[1], 1);
    mbar_init(barO, 1);
    sflag[0] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_o = tmem + 256;       // S buffers at columns 0 and 128

  griddep_wait();
  griddep_launch_dependents();

  int rows_valid = a.rows;
  if (a.rows_dev != nullptr) rows_valid = min(rows_valid, *a.rows_dev);
  const int q_pos0 = a.q_pos0_dev != nullptr ? *a.q_pos0_dev : a.q_pos0;
  const int kv_len = a.kv_len_dev != nullptr ? *a.kv_len_dev : a.kv_len;
  const int row0 = qt * a.tile_pos;
  const int last_row = min(row0 + a.tile_pos, rows_valid) - 1;
  const int kv_hi = last_row >= row0 ? attn_limit(a, q_pos0 + last_row, kv_len) : 0;
  const int ntiles = (kv_hi + 127) / 128;

  const int r_local = r / a.rep;
  const int h_local = r - r_local * a.rep;
  const int q_row = row0 + r_local;
  const bool row_ok = (r_local < a.tile_pos) && (q_row < rows_valid);
  const int head = g * a.rep + h_local;
  const int lim = row_ok ? attn_limit(a, q_pos0 + q_row, kv_len) : 0;
  const int plane = a.kv_plane0 + g;
  const uint32_t idesc = idesc_bf16_f32(128, 128);
  const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;

  auto issue_s = [&](int j) {  // tid 0: S_j = Q K_j^T into S buffer j & 1
    const uint8_t* st = sKV + (j % kAttnStages) * kAttnStageBytes;
    bool ok = (j > 0 || mbar_wait(barQ, 0)) && mbar_wait(&fullKV[j % kAttnStages], (j / kAttnStages) & 1);
    if (!ok) {
      record_error(a.status, DEV_TIMEOUT_TMA);
      sflag[0] = 1;
    } else {
      tc_fence_after();
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(st);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
        umma_bf16(tmem + (j & 1) * 128, sdesc_kmajor_sw128(q_addr + off), sdesc_kmajor_sw128(k_addr + off), idesc,
                  kk != 0 ? 1u : 0u);
      }
    }
    umma_commit(&barS[j & 1]);
  };

  if (tid == 0 && ntiles > 0) {
    const uint32_t qbytes = static_cast<uint32_t>(64 * a.rep * a.tile_pos * 2);
    mbar_expect_tx(barQ, 2 * qbytes);
    tma_load_3d(sQ, &tmQ, barQ, 0, g * a.rep, row0);
    tma_load_3d(sQ + 128 * 128, &tmQ, barQ, 64, g * a.rep, row0);
    for (int j = 0; j < min(kAttnStages, ntiles); ++j) {
      uint8_t* st = sKV + j * kAttnStageBytes;
      const int key0 = j * 128;
      mbar_expect_tx(&fullKV[j], kAttnStageBytes);
      tma_load_3d(st, &tmK, &fullKV[j], 0, key0, plane);
      tma_load_3d(st + 128 * 128, &tmK, &fullKV[j], 64, key0, plane);
      tma_load_3d(st + kAttnKBytes, &tmV, &fullKV[j], key0, 0, plane);
      tma_load_3d(st + kAttnKBytes + 128 * 128, &tmV, &fullKV[j], key0 + 64, 0, plane);
    }
    issue_s(0);
  }

  float o_acc[64];
#pragma unroll
  for (int d = 0; d < 64; ++d) o_acc[d] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;
  bool failed = false;
  int pend_j = ntiles > 0 ? 0 : -1;  // key tile whose S MMA is issued and not yet waited (tid 0)

  for (int j = 0; j < ntiles; ++j) {
    const int s = j % kAttnStages;
    uint8_t* st = sKV + s * kAttnStageBytes;
    const int key0 = j * 128;
    if (!mbar_wait(&barS[j & 1], (j >> 1) & 1)) { record_error(a.status, DEV_TIMEOUT_MMA); sflag[0] = 1; }
    pend_j = -1;
    tc_fence_after();
    __syncthreads();
    if (sflag[0]) { failed = true; break; }
    // next tile's S on the tensor cores while this tile's softmax runs
    if (tid == 0 && j + 1 < ntiles) {
      issue_s(j + 1);
      pend_j = j + 1;
    }

    // This thread's 64 scores of the tile (keys key0 + 64 half ..), read from TMEM once and kept in
    // registers for both passes. The row max is taken over the raw scores and scaled once (the
    // scale is positive and rounding is monotonic, so this is the max of the scaled scores).
    const uint32_t tmem_s = tmem + (j & 1) * 128 + lane_off + half * 64;
    const int k_lo = key0 + half * 64;
    const bool full = k_lo + 64 <= lim;  // every key of this thread's half visible to its row
    float sv[64];
    tmem_ld32x2(tmem_s, sv);
    float tile_max = -INFINITY;
    if (full) {
#pragma unroll
      for (int i = 0; i < 64; ++i) tile_max = fmaxf(tile_max, sv[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i)
        if (k_lo + i < lim) tile_max = fmaxf(tile_max, sv[i]);
    }
    red_m[tid] = tile_max * a.scale_log2;
    __syncthreads();
    tile_max = fmaxf(red_m[r], red_m[r + 128]);
    const float m_new = fmaxf(m_run, tile_max);
    const float alpha = (m_new == -INFINITY) ? 1.0f : exp2f(m_run - m_new);
    const bool live = m_new != -INFINITY;
    float psum = 0.0f;
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      // P = 2^(s scale - m) for 8 keys, packed to bf16 and stored as one 16-byte chunk of the
      // 128-byte-swizzled P tile
      float p[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int i = c8 * 8 + e;
        p[e] = (live && (full || k_lo + i < lim)) ? ex2_ftz(__fmaf_rn(sv[i], a.scale_log2, -m_new)) : 0.0f;
      }
      __align__(16) __nv_bfloat162 pb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        pb[e] = __floats2bfloat162_rn(p[2 * e], p[2 * e + 1]);
        psum += __low2float(pb[e]) + __high2float(pb[e]);
      }
      *reinterpret_cast<uint4*>(sP + sw128_offset(r, half * 64 + c8 * 8, 128)) = *reinterpret_cast<const uint4*>(pb);
    }
    red_s[tid] = psum;
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    l_run = l_run * alpha + (red_s[r] + red_s[r + 128]);
    m_run = m_new;

    if (tid == 0) {
      tc_fence_after();
      const uint32_t p_addr = smem_u32(sP);
      const uint32_t v_addr = smem_u32(st + kAttnKBytes);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
        umma_bf16(tmem_o, sdesc_kmajor_sw128(p_addr + off), sdesc_kmajor_sw128(v_addr + off), idesc,
                  kk != 0 ? 1u : 0u);
      }
      umma_commit(barO);
    }
    if (!mbar_wait(barO, j & 1)) { record_error(a.status, DEV_TIMEOUT_MMA); sflag[0] = 1; }
    tc_fence_after();
#pragma unroll
    for (int cb = 0; cb < 64; cb += 32) {
      float ov[32];
      tmem_ld32(tmem_o + lane_off + half * 64 + cb, ov);
#pragma unroll
      for (int i = 0; i < 32; ++i) o_acc[cb + i] = o_acc[cb + i] * alpha + ov[i];
    }
    // Stage s is free (S_j and PV_j done): refill it with tile j + kAttnStages.
    if (tid == 0 && j + kAttnStages < ntiles && !sflag[0]) {
      const int key1 = (j + kAttnStages) * 128;
      mbar_expect_tx(&fullKV[s], kAttnStageBytes);
      tma_load_3d(st, &tmK, &fullKV[s], 0, key1, plane);
      tma_load_3d(st + 128 * 128, &tmK, &fullKV[s], 64, key1, plane);
      tma_load_3d(st + kAttnKBytes, &tmV, &fullKV[s], key1, 0, plane);
      tma_load_3d(st + kAttnKBytes + 128 * 128, &tmV, &fullKV[s], key1 + 64, 0, plane);
    }
    tc_fence_before();
    __syncthreads();
    if (sflag[0]) { failed = true; break; }
  }

  if (!failed && row_ok) {
    const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
    __nv_bfloat16* dst = a.out + static_cast<size_t>(q_row) * a.nq * 128 + static_cast<size_t>(head) * 128 + half * 64;
#pragma unroll
    for (int d = 0; d < 64; d += 8) {
      __align__(16) __nv_bfloat16 t[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) t[e] = __float2bfloat16_rn(o_acc[d + e] * inv);
      *reinterpret_cast<uint4*>(dst + d) = *reinterpret_cast<const uint4*>(t);
    }
  }
  if (failed && tid == 0) {
    // an S MMA may still be in flight, and loads may still be landing (bounded waits)
    if (pend_j >= 0) mbar_wait(&barS[pend_j & 1], (pend_j >> 1) & 1);
    mbar_wait(barQ, 0);
    for (int s = 0; s < min(kAttnStages, ntiles); ++s) mbar_wait(&fullKV[s], 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace drt
