// Decode-step linear layers: y = x @ W^T for at most 64 activation rows, on tcgen05.
//
// Same transposed product as gemm_swapab_kernel (the weight tile is the M = 128 operand, the
// activation rows are the N operand, the f32 accumulator sits in TMEM with weight row m in lane m),
// specialised for the denoising step, where every linear streams its whole weight once for 32 or
// 64 rows:
//
//  * The MMA width follows the live row count (N = 32 when at most 32 rows are forwarded, else 64).
//  * Split-K over a thread-block cluster of S CTAs along z (S = 1, 2, 4, 8 or 16). Each CTA stages
//    its f32 partial in shared memory as S column slices and sends slice p to CTA p with one bulk
//    shared-to-shared copy (cp.async.bulk ... shared::cluster) that completes on CTA p's receive
//    mbarrier. CTA p waits on that barrier alone, adds the S slices in rank order and runs the
//    epilogue for its columns. Bulk copies move a slice in one operation; per-thread remote loads
//    or stores of the same data measured several times slower on B200. No global workspace, no
//    atomics, and the result does not depend on scheduling.
//  * The stage and receive buffers overlay the weight ring and the activation tile, which are
//    drained once the accumulator is final; one cluster barrier (every CTA past its MMAs) orders
//    the reuse. Most decode shapes then fit in under half of an SM's shared memory, so the next
//    kernel's CTAs can be resident beside this one and stream their weights while it finishes.
//  * The residual epilogue loads the rows it will update before the accumulator is ready.
//
// Weights are prefetched before the programmatic-dependent-launch wait, so their HBM stream
// overlaps the tail of the producing kernel.
#pragma once
#include "gemm.cuh"

namespace drt {

constexpr int kDecRows = 64;                 // activation rows per tile (B operand box)
constexpr int kDecABytes = 128 * 128;        // one K block of the weight tile
constexpr int kDecBBytes = kDecRows * 128;   // one K block of the activation tile
constexpr int kDecMaxKb = 16;                // K blocks of B kept resident per CTA
constexpr int kDecXBytes = 128 * kDecRows * 4;        // one f32 partial tile (receive or stage)

__host__ __device__ inline bool dec_split_supported(int S) { return S == 1 || S == 2 || S == 4 || S == 8 || S == 16; }

// Shared memory: [ring: stages x A block][B: kb_per_split x B block], at least two partial tiles
// long: after the MMAs the first tile holds the outgoing stage and the second the receive buffer
// (later the epilogue scratch).
__host__ __device__ inline size_t dec_ring_bytes(int stages) { return static_cast<size_t>(stages) * kDecABytes; }
__host__ __device__ inline size_t dec_body_bytes(int stages, int kb_per_split) {
  const size_t m = dec_ring_bytes(stages) + static_cast<size_t>(kb_per_split) * kDecBBytes;
  return m > static_cast<size_t>(2 * kDecXBytes) ? m : static_cast<size_t>(2 * kDecXBytes);
}
__host__ __device__ inline size_t dec_smem_bytes(int stages, int kb_per_split) {
  // alignment slack + body + barriers (2 * stages + 3), TMEM slot and flags
  return 1024 + dec_body_bytes(stages, kb_per_split) + static_cast<size_t>(2 * stages + 3) * 8 + 32;
}

__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes, uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_cluster),
               "r"(src_cta), "r"(bytes), "r"(bar_cluster)
               : "memory");
}

// Sum of this CTA's column slice over the S received partials, in rank order. The slice layout is
// [CPR / W][lane][W] per source (W = min(CPR, 4)); S and the MMA width are compile-time so the
// loop is fully unrolled with static indices.
template <int S, int NCOL>
__device__ __forceinline__ void dec_sum_slices(const float* recv, int tid, float* v) {
  constexpr int CPR = NCOL / S;
  constexpr int W = CPR >= 4 ? 4 : 2;
  float buf[S][CPR];
#pragma unroll
  for (int p = 0; p < S; ++p) {
#pragma unroll
    for (int q = 0; q < CPR / W; ++q) {
      const float* src = recv + p * 128 * CPR + (q * 128 + tid) * W;
      if (W == 4) {
        const float4 t = *reinterpret_cast<const float4*>(src);
        buf[p][q * 4] = t.x;
        buf[p][q * 4 + 1] = t.y;
        buf[p][q * 4 + 2] = t.z;
        buf[p][q * 4 + 3] = t.w;
      } else {
        const float2 t = *reinterpret_cast<const float2*>(src);
        buf[p][q * 2] = t.x;
        buf[p][q * 2 + 1] = t.y;
      }
    }
  }
#pragma unroll
  for (int c = 0; c < CPR; ++c) {
    float t = buf[0][c];
#pragma unroll
    for (int p = 1; p < S; ++p) t += buf[p][c];
    v[c] = t;
  }
}

template <int NCOL>
__device__ __forceinline__ void dec_sum_any(int S, const float* recv, int tid, float* v) {
  switch (S) {
    case 2: dec_sum_slices<2, NCOL>(recv, tid, v); break;
    case 4: dec_sum_slices<4, NCOL>(recv, tid, v); break;
    case 8: dec_sum_slices<8, NCOL>(recv, tid, v); break;
    default: dec_sum_slices<16, NCOL>(recv, tid, v); break;
  }
}

__global__ void __launch_bounds__(128, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = a.stages;
  uint8_t* ring = smem;
  uint8_t* sB = ring + dec_ring_bytes(stages);
  float* stage = reinterpret_cast<float*>(smem);
  float* recv = stage + 128 * kDecRows;
  float* xs = recv;  // epilogue scratch, once the received slices are summed
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + dec_body_bytes(stages, a.kb_per_split));
  uint64_t* fullA = bars;
  uint64_t* emptyA = bars + stages;
  uint64_t* fullB = bars + 2 * stages;
  uint64_t* accum = fullB + 1;
  uint64_t* xbar = fullB + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fullB + 3);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] error

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int m0 = blockIdx.x * 128;
  const int kb_total = a.K >> 6;
  const int kb0 = blockIdx.z * a.kb_per_split;
  const int nkb = max(0, min(a.kb_per_split, kb_total - kb0));
  const int S = a.splits;

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&fullA[s], 1);
      mbar_init(&emptyA[s], 1);
    }
    mbar_init(fullB, 1);
    mbar_init(accum, 1);
    mbar_init(xbar, 1);
    flags[0] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  // Weight prefetch first: it depends on nothing the producer kernel writes.
  const int npre = min(stages, nkb);
  uint64_t policy = 0;
  if (tid == 0) {
    policy = l2_policy_evict_first();
    for (int i = 0; i < npre; ++i) {
      mbar_expect_tx(&fullA[i], kDecABytes);
      tma_load_2d_hint(ring + static_cast<size_t>(i) * kDecABytes, &tmA, &fullA[i], (kb0 + i) * 64, m0, policy);
    }
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  griddep_wait();
  int rows_valid = a.rows;
  if (a.rows_dev != nullptr) rows_valid = min(rows_valid, *a.rows_dev);
  rows_valid = max(0, min(rows_valid, kDecRows));
  const int pos0 = a.pos0_dev != nullptr ? *a.pos0_dev : a.pos0;
  const int ncol = rows_valid <= 32 ? 32 : 64;  // MMA N (uniform across the cluster)
  const int cpr = ncol / S;                     // columns owned by each CTA of the cluster
  const uint32_t rank = S > 1 ? cluster_ctarank() : 0u;
  const int c0 = static_cast<int>(rank) * cpr;
  const int nvalid = max(0, min(cpr, rows_valid - c0));
  // Residual epilogue: fetch the rows this CTA will update now, off the critical path.
  float pre[32];
  if (S > 1 && a.epi == EPI_RESID) {
    const int n = m0 + tid;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      pre[i] = i < nvalid ? __ldcg(a.out_f32 + static_cast<size_t>(c0 + i) * a.ld_out + n) : 0.0f;
  }
  if (tid == 0) {
    if (nkb > 0) {
      mbar_expect_tx(fullB, static_cast<uint32_t>(nkb * kDecBBytes));
      for (int i = 0; i < nkb; ++i) tma_load_2d(sB + i * kDecBBytes, &tmB, fullB, (kb0 + i) * 64, 0);
    }
    if (S > 1) mbar_expect_tx(xbar, static_cast<uint32_t>(S * 128 * cpr * 4));
  }
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      for (int i = npre; i < nkb; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&emptyA[s], ((i / stages) - 1) & 1)) { ok = false; break; }
        mbar_expect_tx(&fullA[s], kDecABytes);
        tma_load_2d_hint(ring + static_cast<size_t>(s) * kDecABytes, &tmA, &fullA[s], (kb0 + i) * 64, m0, policy);
      }
      if (!ok) { record_error(a.status, DEV_TIMEOUT_TMA); flags[0] = 1; }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, ncol);
      bool ok = nkb == 0 || mbar_wait(fullB, 0);
      tc_fence_after();
      for (int i = 0; i < nkb && ok; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&fullA[s], (i / stages) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(ring + static_cast<size_t>(s) * kDecABytes);
        const uint32_t b_addr = smem_u32(sB + i * kDecBBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tmem, sdesc_kmajor_sw128(a_addr + kk * 32), sdesc_kmajor_sw128(b_addr + kk * 32), idesc,
                    (i | kk) != 0 ? 1u : 0u);
        umma_commit(&emptyA[s]);
      }
      if (!ok) { record_error(a.status, DEV_TIMEOUT_MMA); flags[0] = 1; }
      umma_commit(accum);
    }
    __syncwarp();
  }

  bool acc_ok = true;
  if (nkb > 0) acc_ok = mbar_wait(accum, 0);
  tc_fence_after();
  if (!acc_ok) { record_error(a.status, DEV_TIMEOUT_EPI); flags[0] = 1; }
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  float acc[64];
  if (acc_ok && nkb > 0) {
    tmem_ld32(lane_addr, acc);
    if (ncol == 64) tmem_ld32(lane_addr + 32, acc + 32);
    else {
#pragma unroll
      for (int c = 32; c < 64; ++c) acc[c] = 0.0f;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 64; ++c) acc[c] = 0.0f;
  }
  if (S == 1) {
    __syncthreads();
    if (flags[0] == 0) {
      gemm_epilogue_chunk(a, acc, 0, min(32, rows_valid), m0, tid, xs, pos0);
      if (rows_valid > 32) gemm_epilogue_chunk(a, acc + 32, 32, rows_valid - 32, m0, tid, xs, pos0);
    }
  } else {
    // Stage the partial as S contiguous slices and send slice p to CTA p. Inside a slice the
    // columns are grouped in units of W = min(cpr, 4): [cpr / W][lane][W], so both the staging
    // stores and the receiver's reads are bank-conflict free. The stage overlays this CTA's
    // drained ring; the receive buffer overlays it too, so nothing is sent before every CTA of the
    // cluster is past its MMAs (the cluster barrier below).
    tc_fence_before();
    __syncthreads();  // every warp is past its TMEM loads
    if (cpr >= 4) {
#pragma unroll
      for (int j = 0; j < 64; j += 4) {
        if (j < ncol) {
          const int p = j / cpr, c = j - p * cpr;
          *reinterpret_cast<float4*>(stage + p * 128 * cpr + ((c >> 2) * 128 + tid) * 4) =
              make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 64; j += 2) {
        if (j < ncol) *reinterpret_cast<float2*>(stage + (j >> 1) * 256 + tid * 2) = make_float2(acc[j], acc[j + 1]);
      }
    }
    fence_proxy_async_smem();
    cluster_sync();  // all stages written, every CTA's ring drained and receive barrier armed
    const uint32_t slice_bytes = static_cast<uint32_t>(128 * cpr * 4);
    if (tid < S) {
      const uint32_t dst = cluster_map(smem_u32(recv) + rank * slice_bytes, static_cast<uint32_t>(tid));
      const uint32_t bar = cluster_map(smem_u32(xbar), static_cast<uint32_t>(tid));
      bulk_copy_to_peer(dst, smem_u32(stage) + tid * slice_bytes, slice_bytes, bar);
    }
    const bool got = mbar_wait(xbar, 0);
    if (!got) { record_error(a.status, DEV_TIMEOUT_EPI); flags[0] = 1; }
    float v[32];
    if (ncol == 32) dec_sum_any<32>(S, recv, tid, v);
    else dec_sum_any<64>(S, recv, tid, v);
    // Every copy into this CTA has landed; once all CTAs pass the final barrier, every copy out of
    // this CTA's stage has too.
    cluster_arrive();
    __syncthreads();  // all slices summed before the epilogue reuses the receive buffer
    if (nvalid > 0 && flags[0] == 0) {
      if (a.epi == EPI_RESID) {
        const int n = m0 + tid;
        const float b = a.bias != nullptr ? a.bias[n] : 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < nvalid)
            a.out_f32[static_cast<size_t>(c0 + i) * a.ld_out + n] = __fadd_rn(pre[i], __fadd_rn(bf16_round(v[i]), b));
      } else {
        gemm_epilogue_chunk(a, v, c0, nvalid, m0, tid, xs, pos0);
      }
    }
    cluster_wait();
  }
  if (flags[0] != 0 && tid == 0) {
    for (int s = 0; s < npre; ++s) mbar_wait(&fullA[s], 0);
    if (nkb > 0) mbar_wait(fullB, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

}  // namespace drt
