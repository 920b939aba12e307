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
//   3. runs a two-pass softmax over its keys with four threads per row, each on a 16-key slice of
//      every sub-tile (pass 1: row max, pass 2: exp2, the bf16 P written over the consumed K
//      sub-tile), in the log2 domain; warps whose 32 rows are all past the live rows skip both
//      passes. One thread's S values (4 sub-tiles x 16 keys) come out of TMEM in one round trip
//      and stay in registers for both passes, so a row costs a few dozen dependent instructions;
//      the softmax, not the K/V stream, set the kernel's time with two threads per row;
//   4. accumulates O = sum_j P_j V_j on the tensor cores into TMEM;
//   5. with one split, normalises and writes bf16. With the splits of a KV head launched as one
//      thread-block cluster (cluster_merge), every CTA pushes its unnormalised f32 rows and (m, l)
//      into the shared memory of the CTA that owns the row (distributed shared memory), and each
//      owner combines its rows over the splits in rank order (rescale by exp2(m_i - max m),
//      normalise, write bf16). Otherwise it writes them to a partial buffer that
//      attn_merge_kernel combines the same way.
// All waits are bounded (common.cuh); on a timeout the CTA records the error and unwinds.
#pragma once
#include "attention.cuh"

namespace drt {

constexpr int kDaMaxSub = 5;                    // 64-key sub-tiles per CTA
constexpr int kDaTmemCols = 512;                // S of kDaMaxSub sub-tiles (64 columns each), power of two
constexpr int kDaRecvStride = 132;              // floats per received row (conflict-free float4 access)
constexpr int kDaMaxSplits = 64;                // CTAs per KV head
constexpr int kDaQBytes = 2 * 128 * 128;        // Q: two 64-d atoms x 128 rows
constexpr int kDaKBytes = 2 * 64 * 128;         // K sub-tile: two 64-d atoms x 64 keys
constexpr int kDaVBytes = 128 * 128;            // V^T sub-tile: 128 d rows x 64 keys
constexpr int kDaSubBytes = kDaKBytes + kDaVBytes;
constexpr int kDaThreads = 512;                  // four threads per UMMA row
// Q | sub-tiles | row-statistics exchange | barriers
constexpr size_t kDaBodyBytes = kDaQBytes + static_cast<size_t>(kDaMaxSub) * kDaSubBytes;
constexpr size_t kDaRedFloats = 8 * 128;        // softmax row statistics: [4 slices][128] maxima, then sums
constexpr size_t kDaSmemBytes = 1024 + kDaBodyBytes + kDaRedFloats * 4 + 256;
// The cluster merge's receive buffer ([S][R] rows plus (m, l), S R <= 128 + 15) overlays the sub-tiles.
static_assert((128 + 15) * (kDaRecvStride + 2) * 4 <= kDaMaxSub * kDaSubBytes, "receive buffer exceeds the sub-tile area");

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
  int cluster_merge;      // splits > 1 launched as one cluster per KV head: merge in shared memory
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

// Columns [c, c + 16) of this thread's TMEM lane in each of the four 64-column blocks at taddr
// (32x32b.x16 shape): v[16 j + i] = column 64 j + i. One wait for all four loads, in the same
// statement, so no use of the registers can be scheduled before the data lands.
__device__ __forceinline__ void tmem_ld16x4(uint32_t taddr, float* v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%65];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47}, [%66];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%67];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr), "r"(taddr + 64), "r"(taddr + 128), "r"(taddr + 192)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// Columns [c, c + 16) of this thread's TMEM lane at taddr, with the wait.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(kDaThreads, 1)
    attn_decode_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK64,
                       const __grid_constant__ CUtensorMap tmV, const DecAttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sSub = smem + kDaQBytes;  // [kDaMaxSub][K | V^T]
  float* red = reinterpret_cast<float*>(smem + kDaBodyBytes);  // [4][128] row maxima, [4][128] row sums
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
  // The host sizes `splits` so that no CTA gets more than kDaMaxSub sub-tiles; a mismatch is reported
  // instead of dropping keys (the loads stay within the CTA's kDaMaxSub slots either way).
  if (sub1 - sub0 > kDaMaxSub && tid == 0) record_error(a.status, DEV_BAD_GEOMETRY);
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
    tmem_alloc(tmem_slot, kDaTmemCols);
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
  const int lane = tid & 31;
  const int quarter = warp & 3;  // TMEM lanes [32 quarter, 32 quarter + 32): rows of this warp
  const int slice = warp >> 2;   // keys [16 slice, 16 slice + 16) of every sub-tile, output dims [32 slice, +32)
  const int r = quarter * 32 + lane;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const int pos = r / a.rep;
  const bool row_ok = r < rows_total;
  const bool warp_live = nt > 0 && quarter * 32 < rows_total;  // warp-uniform
  const int lim = row_ok ? da_limit(a, q_pos0 + pos, kv_len) : 0;
  if (nt > 0 && !mbar_wait(barS, 0)) { record_error(a.status, DEV_TIMEOUT_MMA); flags[0] = 1; }
  tc_fence_after();

  // ---- pass 1: row max of the raw scores over this thread's keys (the scale is positive, so the
  // max of the scaled scores is the scaled max, rounding being monotonic)
  float sv[16 * kDaMaxSub];
  float mpart = -INFINITY;
  if (warp_live) {
    tmem_ld16x4(tmem + lane_off + slice * 16, sv);
    if (nt > 4) tmem_ld16(tmem + lane_off + 256 + slice * 16, sv + 64);
#pragma unroll
    for (int j = 0; j < kDaMaxSub; ++j) {
      const int k0 = (sub0 + j) * 64 + slice * 16;
      if (j < nt) {
        if (k0 + 16 <= lim) {
#pragma unroll
          for (int i = 0; i < 16; ++i) mpart = fmaxf(mpart, sv[j * 16 + i]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (k0 + i < lim) mpart = fmaxf(mpart, sv[j * 16 + i]);
        }
      }
    }
  }
  red[slice * 128 + r] = mpart;
  __syncthreads();
  const float m = fmaxf(fmaxf(red[r], red[128 + r]), fmaxf(red[256 + r], red[384 + r])) * a.scale_log2;
  // ---- pass 2: P = exp2(s scale - m) as bf16 over the consumed K sub-tile; partial row sums
  float lpart = 0.0f;
  if (warp_live) {
#pragma unroll
    for (int j = 0; j < kDaMaxSub; ++j) {
      if (j < nt) {
        const int k0 = (sub0 + j) * 64 + slice * 16;
        const bool full = k0 + 16 <= lim;
        float p[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          p[i] = (full || k0 + i < lim) ? ex2_ftz(__fmaf_rn(sv[j * 16 + i], a.scale_log2, -m)) : 0.0f;
        __align__(16) __nv_bfloat162 t[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = __floats2bfloat162_rn(p[2 * i], p[2 * i + 1]);
#pragma unroll
        for (int i = 0; i < 8; ++i) lpart += __low2float(t[i]) + __high2float(t[i]);
        uint8_t* sP = sSub + static_cast<size_t>(j) * kDaSubBytes;  // [128 rows][64 keys] SW128
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int chunk = (slice * 2 + h) ^ (r & 7);
          *reinterpret_cast<uint4*>(sP + r * 128 + chunk * 16) = *reinterpret_cast<const uint4*>(t + h * 4);
        }
      }
    }
  }
  red[512 + slice * 128 + r] = lpart;
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  const float l = ((red[512 + r] + red[640 + r]) + red[768 + r]) + red[896 + r];

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
  float o[32];
  if (warp_live) {
    tmem_ld32(tmem + lane_off + slice * 32, o);
  } else {
#pragma unroll
    for (int d = 0; d < 32; ++d) o[d] = 0.0f;
  }
  const float m_out = nt > 0 ? m : -INFINITY;
  const float l_out = nt > 0 ? l : 0.0f;

  if (a.cluster_merge && S > 1) {
    // Every CTA's loads and UMMAs are done before any peer writes into its sub-tile area (which
    // the receive buffer overlays): settle this CTA's copies, arrive, then wait for all.
    if (flags[0] != 0 && tid == 0) {
      if (nt > 0) mbar_wait(barQ, 0);
      for (int j = 0; j < nt; ++j) mbar_wait(&barKV[j], 0);
    }
    tc_fence_before();
    __syncthreads();
    cluster_arrive();
    const int R = (rows_total + S - 1) / S;                      // rows owned by each CTA
    float* recv = reinterpret_cast<float*>(sSub);                // [S sources][R][kDaRecvStride]
    float* recv_ml = recv + static_cast<size_t>(S) * R * kDaRecvStride;  // [S][R][2]
    const bool failed = flags[0] != 0;
    cluster_wait();
    if (row_ok) {
      const uint32_t rank = cluster_ctarank();
      const uint32_t owner = static_cast<uint32_t>(r / R);
      const int slot = static_cast<int>(rank) * R + (r % R);
      const uint32_t dst = cluster_map(smem_u32(recv + static_cast<size_t>(slot) * kDaRecvStride + slice * 32), owner);
#pragma unroll
      for (int d = 0; d < 32; d += 4)
        st_cluster_f32x4(dst + d * 4, failed ? make_float4(0.f, 0.f, 0.f, 0.f) : make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]));
      if (slice == 0)
        st_cluster_f32x2(cluster_map(smem_u32(recv_ml + slot * 2), owner), failed ? -INFINITY : m_out, failed ? 0.0f : l_out);
    }
    cluster_sync();
    // Owner: rows [rank R, rank R + R), one (row, 4 output dims) item per thread.
    const int rank = static_cast<int>(cluster_ctarank());
    for (int item = tid; item < R * 32; item += kDaThreads) {
      const int lr = item >> 5, c4 = item & 31;
      const int row = rank * R + lr;
      if (row >= rows_total) break;
      float mx = -INFINITY;
      for (int p = 0; p < S; ++p) {
        const float2 ml = *reinterpret_cast<const float2*>(recv_ml + (p * R + lr) * 2);
        if (ml.y > 0.0f) mx = fmaxf(mx, ml.x);
      }
      float L = 0.0f;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int p = 0; p < S; ++p) {
        const float2 ml = *reinterpret_cast<const float2*>(recv_ml + (p * R + lr) * 2);
        const float w = ml.y > 0.0f ? exp2f(ml.x - mx) : 0.0f;
        const float4 v = *reinterpret_cast<const float4*>(recv + static_cast<size_t>(p * R + lr) * kDaRecvStride + c4 * 4);
        L += ml.y * w;
        acc[0] += v.x * w;
        acc[1] += v.y * w;
        acc[2] += v.z * w;
        acc[3] += v.w * w;
      }
      const int rpos = row / a.rep;
      const int head = g * a.rep + (row - rpos * a.rep);
      __align__(8) __nv_bfloat16 t[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) t[e] = __float2bfloat16_rn(L > 0.0f ? acc[e] / L : 0.0f);
      *reinterpret_cast<uint2*>(a.out + (static_cast<size_t>(rpos) * a.nq + head) * 128 + c4 * 4) =
          *reinterpret_cast<const uint2*>(t);
    }
  } else if (row_ok && flags[0] == 0) {
    if (S == 1) {
      const float inv = l_out > 0.0f ? 1.0f / l_out : 0.0f;
      const int head = g * a.rep + (r - pos * a.rep);
      __nv_bfloat16* dst = a.out + (static_cast<size_t>(pos) * a.nq + head) * 128 + slice * 32;
#pragma unroll
      for (int d = 0; d < 32; d += 8) {
        __align__(16) __nv_bfloat16 t[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) t[e] = __float2bfloat16_rn(o[d + e] * inv);
        *reinterpret_cast<uint4*>(dst + d) = *reinterpret_cast<const uint4*>(t);
      }
    } else {
      // dims-major so that each store of a warp (32 consecutive rows, one dim) fills one 128-byte line
      const size_t prow = (static_cast<size_t>(g) * S + split) * 128 + r;
      float* dst = a.part_o + prow * 128 + slice * 32;
#pragma unroll
      for (int d = 0; d < 32; d += 4) *reinterpret_cast<float4*>(dst + d) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
      if (slice == 0) *reinterpret_cast<float2*>(a.part_ml + prow * 2) = make_float2(m_out, l_out);
    }
  }
  if (flags[0] != 0 && tid == 0) {
    if (nt > 0) mbar_wait(barQ, 0);
    for (int j = 0; j < nt; ++j) mbar_wait(&barKV[j], 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kDaTmemCols);
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
