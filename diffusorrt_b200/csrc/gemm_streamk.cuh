// Stream-K linear for decode-shaped activations (at most 128 rows) whose output tiles leave SMs
// idle: Dream-7B's down_proj over a decode window is 28 weight tiles of 128 rows with K = 18944,
// which one CTA per tile would stream on 28 of the 148 SMs.
//
// The T x KB (tile, K block) iterations are split into G equal contiguous ranges, one per CTA of a
// persistent grid (G <= SMs, one CTA per SM, so every CTA is resident). Iterations run tile by
// tile. A CTA's range cuts at most its first tile (a tail: K blocks from the middle to the end)
// and its last (a head: K blocks from 0); every tile between is whole. Segments run in order, so a
// tail is finished first and a head last:
//   * a tail's f32 partial goes to this CTA's workspace slot, then its ready flag is raised;
//   * a head's CTA owns the tile: it waits (bounded) for the flags of the CTAs that cover the rest
//     of the tile (the next ones in order), adds their partials to its accumulator in CTA order
//     (a fixed order: the result does not depend on timing), resets those flags for the next
//     launch, and runs the linear's epilogue.
// The ring's stage counter and the accumulator barrier's phase carry across segments; each
// segment's first UMMA overwrites the accumulator. Epilogues: EPI_STORE_F32, EPI_STORE_RAW,
// EPI_RESID, EPI_SWIGLU (a tile's owner holds all 128 weight rows of the tile, gate and up).
#pragma once
#include "gemm.cuh"

namespace drt {

template <int BN, int KS>
__global__ void __launch_bounds__(128, 1)
    gemm_streamk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmArgs a) {
  using Cfg = GemmCfg<BN, KS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  const int stages = a.stages;
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + Cfg::body_bytes(stages));
  uint64_t* full = bars;
  uint64_t* empty = bars + stages;
  uint64_t* accum = bars + 2 * stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  // [0] error, [1] ring stages issued, [2] ring stages consumed, [3] an owner's wait ran out
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int tiles_m = a.n_out >> 7;
  const int tiles_n = (a.rows + BN - 1) / BN;
  const int KB = a.K >> 6;
  const long long total = static_cast<long long>(tiles_m) * tiles_n * KB;
  const long long it0 = total * c / G, it1 = total * (c + 1) / G;

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    flags[3] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  int rows_valid = a.rows;
  if (a.rows_dev != nullptr) rows_valid = min(rows_valid, *a.rows_dev);
  const int pos0 = a.pos0_dev != nullptr ? *a.pos0_dev : a.pos0;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const uint64_t policy = l2_policy_evict_first();  // each weight tile is read by one CTA
  float* xs = reinterpret_cast<float*>(ring);  // epilogue scratch over the drained ring
  int gi = 0;   // ring stages used so far (both lanes follow the same sequence)
  int seg = 0;  // segments finished (phase of the accumulator barrier)
  for (long long it = it0; it < it1;) {
    const int t = static_cast<int>(it / KB);
    const int ka = static_cast<int>(it - static_cast<long long>(t) * KB);
    const int kend = static_cast<int>(min(static_cast<long long>(KB), it1 - static_cast<long long>(t) * KB));
    const int nkb = kend - ka;
    const int nsb = (nkb + KS - 1) / KS;
    const int m0 = (t / tiles_n) * 128, n0 = (t % tiles_n) * BN;
    if (warp == 0) {
      if (lane == 0) {
        bool ok = flags[0] == 0;
        for (int i = 0; i < nsb && ok; ++i) {
          const int g = gi + i, s = g % stages;
          const int nk = min(KS, nkb - i * KS);
          if (g >= stages && !mbar_wait(&empty[s], ((g / stages) - 1) & 1)) { ok = false; break; }
          uint8_t* st = ring + static_cast<size_t>(s) * Cfg::kStageBytes;
          mbar_expect_tx(&full[s], static_cast<uint32_t>(nk * (Cfg::kABytes + Cfg::kBBytes)));
          for (int j = 0; j < nk; ++j) {
            const int k = (ka + i * KS + j) * 64;
            tma_load_2d_hint(st + j * Cfg::kABytes, &tmA, &full[s], k, m0, policy);
            tma_load_2d(st + KS * Cfg::kABytes + j * Cfg::kBBytes, &tmB, &full[s], k, n0);
          }
          flags[1] = g + 1;
        }
        if (!ok) { record_error(a.status, DEV_TIMEOUT_TMA); flags[0] = 1; }
      }
      __syncwarp();
    } else if (warp == 1) {
      if (lane == 0) {
        const uint32_t idesc = idesc_bf16_f32(128, BN);
        bool ok = true;
        for (int i = 0; i < nsb; ++i) {
          const int g = gi + i, s = g % stages;
          const int nk = min(KS, nkb - i * KS);
          if (!mbar_wait(&full[s], (g / stages) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + static_cast<size_t>(s) * Cfg::kStageBytes);
          const uint32_t b_addr = a_addr + KS * Cfg::kABytes;
#pragma unroll
          for (int j = 0; j < KS; ++j) {
            if (j < nk) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_bf16(tmem, sdesc_kmajor_sw128(a_addr + j * Cfg::kABytes + kk * 32),
                          sdesc_kmajor_sw128(b_addr + j * Cfg::kBBytes + kk * 32), idesc, (i | j | kk) != 0 ? 1u : 0u);
            }
          }
          umma_commit(&empty[s]);
          flags[2] = g + 1;
        }
        if (!ok) { record_error(a.status, DEV_TIMEOUT_MMA); flags[0] = 1; }
        umma_commit(accum);
      }
      __syncwarp();
    }
    if (!mbar_wait(accum, seg & 1)) { record_error(a.status, DEV_TIMEOUT_EPI); flags[0] = 1; }
    tc_fence_after();
    __syncthreads();
    const bool failed = flags[0] != 0;
    if (ka != 0) {
      // tail: this CTA's partial to its workspace slot ([column][row]: coalesced), then the flag
      float* part = a.sk_part + static_cast<size_t>(c) * BN * 128;
      if (!failed) {
#pragma unroll 1
        for (int cb = 0; cb < BN; cb += 32) {
          float v[32];
          tmem_ld32(lane_addr + cb, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) part[static_cast<size_t>(cb + i) * 128 + tid] = v[i];
        }
      }
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        st_release_gpu_u32(reinterpret_cast<unsigned int*>(a.sk_flag + c), 1u);
      }
    } else {
      // head: wait for the CTAs covering the rest of the tile, add their partials in CTA order
      const long long last_it = static_cast<long long>(t) * KB + KB - 1;
      const int c_last = static_cast<int>(((last_it + 1) * G + total - 1) / total) - 1;
      if (tid == 0) {
        int bad = 0;
        for (int q = c + 1; q <= c_last && !bad; ++q) {
          const uint64_t t0 = globaltimer_ns();
          while (ld_acquire_gpu_u32(reinterpret_cast<const unsigned int*>(a.sk_flag + q)) == 0u) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) { bad = 1; break; }
          }
        }
        if (bad) { record_error(a.status, DEV_TIMEOUT_EPI); flags[0] = 1; }
        flags[3] = bad;
      }
      __syncthreads();
      const int ncol_valid = max(0, min(BN, rows_valid - n0));
      if (!flags[3] && !failed) {
#pragma unroll 1
        for (int cb = 0; cb < ncol_valid; cb += 32) {
          float v[32];
          tmem_ld32(lane_addr + cb, v);
          for (int q = c + 1; q <= c_last; ++q) {
            const float* part = a.sk_part + static_cast<size_t>(q) * BN * 128;
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] += __ldcg(part + static_cast<size_t>(cb + i) * 128 + tid);
          }
          gemm_epilogue_chunk(a, v, n0 + cb, min(32, ncol_valid - cb), m0, tid, xs, pos0);
        }
      }
      tc_fence_before();
      __syncthreads();
      if (tid == 0)
        for (int q = c + 1; q <= c_last; ++q) a.sk_flag[q] = 0;  // every partial of this tile is consumed
    }
    tc_fence_after();
    gi += nsb;
    ++seg;
    it = static_cast<long long>(t) * KB + kend;
  }
  if (flags[0] != 0 && tid == 0) {
    // a wait ran out: let this CTA's own copies land before its shared memory goes away
    for (int g = flags[2]; g < flags[1]; ++g) mbar_wait(&full[g % stages], (g / stages) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace drt
