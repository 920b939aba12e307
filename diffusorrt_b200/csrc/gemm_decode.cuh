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
constexpr int kDecPreStages = 2;             // weight K blocks requested before the dependency wait
constexpr int kDecXBytes = 128 * kDecRows * 4;        // one f32 partial tile (receive or stage)

// Quantized instantiations (QB = 4: 4-bit affine, QB = 8: int8 weight-only as an affine form): every
// packed tile of the CTA's K slice is resident (dec_p_bytes(QB) each), the dequantized bf16 weight
// tiles go through a ring of kDecQStages A blocks.
__host__ __device__ constexpr int dec_p_bytes(int qb) { return 128 * 64 * qb / 8; }  // 128 rows x 64 packed inputs
constexpr int kDecQStages = 3;
constexpr int kDecQMaxKb = 8;         // K blocks per CTA for the quantized instantiation

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
// Quantized: [A ring kDecQStages][B kb][packed kb][scale kb x 128 f32][bias kb x 128 f32], at least two
// partial tiles long (stage and receive overlays).
__host__ __device__ inline size_t dec_q_body_bytes(int kb_per_split, int qb) {
  const size_t m = static_cast<size_t>(kDecQStages) * kDecABytes +
                   static_cast<size_t>(kb_per_split) * (kDecBBytes + dec_p_bytes(qb) + 2 * 128 * 4);
  return m > static_cast<size_t>(2 * kDecXBytes) ? m : static_cast<size_t>(2 * kDecXBytes);
}
__host__ __device__ inline size_t dec_q_smem_bytes(int kb_per_split, int qb) {
  return 1024 + dec_q_body_bytes(kb_per_split, qb) + static_cast<size_t>(2 * kDecQStages + 4) * 8 + 32;
}

__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes, uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_cluster),
               "r"(src_cta), "r"(bytes), "r"(bar_cluster)
               : "memory");
}

// Decode epilogues, written in phases (every shared-memory read of a phase is issued before the
// first dependent use, and every global store comes last) over a compile-time number of columns
// CPR with no per-column guards except on the stores, so the few warps of a CTA keep many
// independent operations in flight; results are those of gemm_epilogue_chunk.
//
// QKV tile, columns [c0, c0 + nc) of this CTA's slice (v[i] = accumulator of column c0 + i,
// nc <= CPR): q / k rows get bias, the per-row RMSNorm over the head (QK-norm) and RoPE; v rows
// are written transposed into the V^T cache. rope_c / rope_s hold this thread's RoPE factors.
template <int CPR, bool RND>
__device__ __forceinline__ void dec_epilogue_qkv(const GemmArgs& a, const float* v, int c0, int nc, int m0, int tid,
                                                 float* xs, int pos0, const float* rope_c, const float* rope_s) {
  const int n = m0 + tid;
  const float b = a.bias != nullptr ? a.bias[n] : 0.0f;
  const int tile = m0 >> 7;
  const bool is_q = tile < a.nq;
  const bool is_k = !is_q && tile < a.nq + a.nkv;
  float val[CPR];
#pragma unroll
  for (int i = 0; i < CPR; ++i) val[i] = __fadd_rn(out_round<RND>(v[i]), b);
  if (!is_q && !is_k) {
    // V^T[g][d][pos], contiguous along pos: this thread's feature row, nc consecutive positions.
    const int g = tile - a.nq - a.nkv;
    __nv_bfloat16* dst = a.vtcache + (static_cast<size_t>(g) * 128 + tid) * a.max_seq + pos0 + c0;
    if (CPR % 8 == 0 && nc == CPR && ((pos0 + c0) & 7) == 0) {
#pragma unroll
      for (int q = 0; q < CPR / 8; ++q) {
        __align__(16) __nv_bfloat16 t[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) t[e] = __float2bfloat16_rn(val[q * 8 + e]);
        *reinterpret_cast<uint4*>(dst + q * 8) = *reinterpret_cast<const uint4*>(t);
      }
    } else {
#pragma unroll
      for (int i = 0; i < CPR; ++i)
        if (i < nc) dst[i] = __float2bfloat16_rn(val[i]);
    }
    return;
  }
  const float* nw = is_q ? a.qnorm_w : a.knorm_w;
  const int warp = tid >> 5, lane = tid & 31;
  const int partner = tid ^ 64;
  const float w_self = nw != nullptr ? nw[tid] : 1.0f;
  const float w_part = nw != nullptr ? nw[partner] : 1.0f;
  float* rs = xs + 32 * 128;  // per-row scales
  float* part = rs + 32;        // [4 warps][32 rows]
#pragma unroll
  for (int i = 0; i < CPR; ++i) xs[i * 128 + tid] = val[i];
  if (nw != nullptr) {
    float sq[CPR];
#pragma unroll
    for (int i = 0; i < CPR; ++i) sq[i] = __fmul_rn(val[i], val[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int i = 0; i < CPR; ++i) sq[i] += __shfl_xor_sync(0xffffffffu, sq[i], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < CPR; ++i) part[warp * 32 + i] = sq[i];
    }
  }
  __syncthreads();
  if (nw != nullptr && tid < CPR) {
    const float ss = __fadd_rn(__fadd_rn(__fadd_rn(part[tid], part[32 + tid]), part[64 + tid]), part[96 + tid]);
    rs[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), a.eps)));
  }
  __syncthreads();
  float xp[CPR], sc[CPR];
#pragma unroll
  for (int i = 0; i < CPR; ++i) {
    xp[i] = xs[i * 128 + partner];
    sc[i] = nw != nullptr ? rs[i] : 1.0f;
  }
  __nv_bfloat16 outv[CPR];
#pragma unroll
  for (int i = 0; i < CPR; ++i) {
    float x = val[i], y = xp[i];
    if (nw != nullptr) {
      x = __fmul_rn(__fmul_rn(x, sc[i]), w_self);
      y = __fmul_rn(__fmul_rn(y, sc[i]), w_part);
    }
    const float rot = tid < 64 ? -y : y;
    outv[i] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(x, rope_c[i]), __fmul_rn(rot, rope_s[i])));
  }
  const int head = is_q ? tile : tile - a.nq;
#pragma unroll
  for (int i = 0; i < CPR; ++i) {
    if (i < nc) {
      if (is_q) a.out_bf16[(static_cast<size_t>(c0 + i) * a.nq + head) * 128 + tid] = outv[i];
      else a.kcache[(static_cast<size_t>(head) * a.max_seq + pos0 + c0 + i) * 128 + tid] = outv[i];
    }
  }
}

// SwiGLU tile (lanes 0..63 gate rows j0 + f, lanes 64..127 up rows j0 + f of the same features):
// act[c0 + i, j0 + f] = bf16(silu(g) * u). Both halves of the CTA work: thread t takes feature
// t & 63 for the columns of parity t >> 6.
template <int CPR, bool RND>
__device__ __forceinline__ void dec_epilogue_swiglu(const GemmArgs& a, const float* v, int c0, int nc, int m0, int tid,
                                                    float* xs) {
  const float b = a.bias != nullptr ? a.bias[m0 + tid] : 0.0f;
#pragma unroll
  for (int i = 0; i < CPR; ++i) xs[i * 128 + tid] = __fadd_rn(out_round<RND>(v[i]), b);
  __syncthreads();
  constexpr int H = CPR / 2;
  const int f = tid & 63, par = tid >> 6;
  float g[H], u[H];
#pragma unroll
  for (int k = 0; k < H; ++k) {
    g[k] = xs[(2 * k + par) * 128 + f];
    u[k] = xs[(2 * k + par) * 128 + 64 + f];
  }
  __nv_bfloat16 act[H];
#pragma unroll
  for (int k = 0; k < H; ++k) {
    const float sig = 1.0f / (1.0f + expf(-g[k]));
    act[k] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(g[k], sig), u[k]));
  }
  const int j0 = m0 >> 1;
#pragma unroll
  for (int k = 0; k < H; ++k) {
    const int i = 2 * k + par;
    if (i < nc) a.out_bf16[static_cast<size_t>(c0 + i) * a.ld_out + j0 + f] = act[k];
  }
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


// Shared-memory carve-up of one decode-linear CTA.
struct DecSmem {
  uint8_t* ring;
  uint8_t* sB;
  uint8_t* sP;      // quantized: packed tiles [kb][128 rows][64 * QB / 8 bytes]
  float* qsc;       // quantized: [kb][128] scales of this CTA's rows
  float* qbi;       // quantized: [kb][128] biases
  uint64_t* fullP;  // quantized: all packed tiles landed
  float* stage;
  float* recv;
  float* xs;
  uint64_t* fullA;
  uint64_t* emptyA;
  uint64_t* fullB;
  uint64_t* accum;
  uint64_t* xbar;
  int* flags;
};

// Everything after the dependency wait, for a compile-time epilogue EPI, split-K factor S and MMA
// width NCOL: activation load, weight ring, UMMA, split-K exchange and epilogue.
template <int EPI, int S, int NCOL, int QB>
__device__ __forceinline__ void dec_run(const CUtensorMap* tmA, const CUtensorMap* tmB, const GemmArgs& a, const DecSmem& sm,
                                        uint32_t tmem, int m0, int kb0, int nkb, int npre, int stages, uint64_t policy,
                                        int rows_valid, int pos0) {
  constexpr int CPR = NCOL / S;  // columns owned by each CTA of the cluster
  constexpr bool QUANT = QB != 0;
  // Output rounding: the bf16 contract rounds every linear output to bf16, and so does int8
  // weight-only (bf16 activations); the 4-bit quantized-matmul contract keeps f32 outputs.
  constexpr bool RND = QB != 4;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = S > 1 ? cluster_ctarank() : 0u;
  const int c0 = static_cast<int>(rank) * CPR;
  const int nvalid = max(0, min(CPR, rows_valid - c0));
  // Epilogue inputs that do not depend on the accumulator are fetched now, off the critical path:
  // the residual rows this CTA will update, or the RoPE factors of its Q/K rows.
  float pre[CPR], pre2[CPR];
  if constexpr (S > 1 && EPI == EPI_RESID) {
    const int n = m0 + tid;
#pragma unroll
    for (int i = 0; i < CPR; ++i) pre[i] = i < nvalid ? __ldcg(a.out_f32 + static_cast<size_t>(c0 + i) * a.ld_out + n) : 0.0f;
  }
  if constexpr (S > 1 && EPI == EPI_QKV) {
    if ((m0 >> 7) < a.nq + a.nkv) {
#pragma unroll
      for (int i = 0; i < CPR; ++i) {
        const size_t idx = static_cast<size_t>(pos0 + c0 + i) * 64 + (tid & 63);
        pre[i] = i < nvalid ? __ldg(a.rope_cos + idx) : 0.0f;
        pre2[i] = i < nvalid ? __ldg(a.rope_sin + idx) : 0.0f;
      }
    }
  }
  if (tid == 0) {
    if (nkb > 0) {
      mbar_expect_tx(sm.fullB, static_cast<uint32_t>(nkb * kDecBBytes));
      for (int i = 0; i < nkb; ++i) tma_load_2d(sm.sB + i * kDecBBytes, tmB, sm.fullB, (kb0 + i) * 64, 0);
    }
    if constexpr (S > 1) mbar_expect_tx(sm.xbar, static_cast<uint32_t>(S * 128 * CPR * 4));
  }
  griddep_launch_dependents();

  if constexpr (QUANT) {
    // Dequantize group g of this CTA's rows into ring slot g % kDecQStages (thread t: row t), then one
    // lane issues its UMMAs; the next group's dequantization overlaps them.
    bool ok = nkb == 0 || (mbar_wait(sm.fullP, 0) && mbar_wait(sm.fullB, 0));
    ok = __syncthreads_and(ok) != 0;  // uniform across the CTA, so every barrier below is reached by all
    for (int g = 0; g < nkb && ok; ++g) {
      const int slot = g % kDecQStages;
      bool ready = g < kDecQStages || mbar_wait(&sm.emptyA[slot], ((g / kDecQStages) - 1) & 1);
      constexpr int kRowBytes = 64 * QB / 8;  // packed bytes of one row's group
      const uint8_t* prow = sm.sP + g * dec_p_bytes(QB) + tid * kRowBytes;
      uint32_t pw[kRowBytes / 4];
#pragma unroll
      for (int w4 = 0; w4 < kRowBytes / 16; ++w4) {
        const uint4 p = *reinterpret_cast<const uint4*>(prow + w4 * 16);
        pw[w4 * 4] = p.x;
        pw[w4 * 4 + 1] = p.y;
        pw[w4 * 4 + 2] = p.z;
        pw[w4 * 4 + 3] = p.w;
      }
      const float sc = sm.qsc[g * 128 + tid], bi = sm.qbi[g * 128 + tid];
      uint8_t* arow = sm.ring + static_cast<size_t>(slot) * kDecABytes + tid * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 8 inputs per 16-byte chunk
        __align__(16) __nv_bfloat16 t[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          // 4-bit: input 8c + e is nibble e of word c; 8-bit: byte e % 4 of word 2c + e / 4
          const uint32_t qi = QB == 4 ? (pw[c] >> (4 * e)) & 15u : (pw[2 * c + e / 4] >> (8 * (e % 4))) & 255u;
          t[e] = __float2bfloat16_rn(__fmaf_rn(sc, static_cast<float>(qi), bi));
        }
        *reinterpret_cast<uint4*>(arow + ((c ^ (tid & 7)) * 16)) = *reinterpret_cast<const uint4*>(t);
      }
      fence_proxy_async_smem();
      ok = __syncthreads_and(ready) != 0;
      if (!ok) break;
      if (warp == 1 && lane == 0) {
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(128, NCOL);
        const uint32_t a_addr = smem_u32(sm.ring + static_cast<size_t>(slot) * kDecABytes);
        const uint32_t b_addr = smem_u32(sm.sB + g * kDecBBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tmem, sdesc_kmajor_sw128(a_addr + kk * 32), sdesc_kmajor_sw128(b_addr + kk * 32), idesc,
                    (g | kk) != 0 ? 1u : 0u);
        umma_commit(&sm.emptyA[slot]);
      }
    }
    if (!ok) { record_error(a.status, DEV_TIMEOUT_MMA); sm.flags[0] = 1; }
    if (warp == 1 && lane == 0) umma_commit(sm.accum);
    __syncwarp();
  } else {
  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      for (int i = npre; i < nkb; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&sm.emptyA[s], ((i / stages) - 1) & 1)) { ok = false; break; }
        mbar_expect_tx(&sm.fullA[s], kDecABytes);
        tma_load_2d_hint(sm.ring + static_cast<size_t>(s) * kDecABytes, tmA, &sm.fullA[s], (kb0 + i) * 64, m0, policy);
      }
      if (!ok) { record_error(a.status, DEV_TIMEOUT_TMA); sm.flags[0] = 1; }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, NCOL);
      bool ok = nkb == 0 || mbar_wait(sm.fullB, 0);
      tc_fence_after();
      for (int i = 0; i < nkb && ok; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&sm.fullA[s], (i / stages) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sm.ring + static_cast<size_t>(s) * kDecABytes);
        const uint32_t b_addr = smem_u32(sm.sB + i * kDecBBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tmem, sdesc_kmajor_sw128(a_addr + kk * 32), sdesc_kmajor_sw128(b_addr + kk * 32), idesc,
                    (i | kk) != 0 ? 1u : 0u);
        umma_commit(&sm.emptyA[s]);
      }
      if (!ok) { record_error(a.status, DEV_TIMEOUT_MMA); sm.flags[0] = 1; }
      umma_commit(sm.accum);
    }
    __syncwarp();
  }
  }

  bool acc_ok = true;
  if (nkb > 0) acc_ok = mbar_wait(sm.accum, 0);
  tc_fence_after();
  if (!acc_ok) { record_error(a.status, DEV_TIMEOUT_EPI); sm.flags[0] = 1; }
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  float acc[NCOL];
  if (acc_ok && nkb > 0) {
#pragma unroll
    for (int cb = 0; cb < NCOL; cb += 32) tmem_ld32(lane_addr + cb, acc + cb);
  } else {
#pragma unroll
    for (int c = 0; c < NCOL; ++c) acc[c] = 0.0f;
  }
  if constexpr (S == 1) {
    __syncthreads();
    if (sm.flags[0] == 0) {
      gemm_epilogue_chunk_t<EPI, RND>(a, acc, 0, min(32, rows_valid), m0, tid, sm.xs, pos0);
      if constexpr (NCOL == 64)
        if (rows_valid > 32) gemm_epilogue_chunk_t<EPI, RND>(a, acc + 32, 32, rows_valid - 32, m0, tid, sm.xs, pos0);
    }
  } else {
    // Stage the partial as S contiguous slices and send slice p to CTA p. Inside a slice the
    // columns are grouped in units of W = min(CPR, 4): [CPR / W][lane][W], so both the staging
    // stores and the receiver's reads are bank-conflict free. The stage overlays this CTA's
    // drained ring; the receive buffer overlays it too, so nothing is sent before every CTA of the
    // cluster is past its MMAs (the cluster barrier below).
    tc_fence_before();
    __syncthreads();  // every warp is past its TMEM loads
    if constexpr (CPR >= 4) {
#pragma unroll
      for (int j = 0; j < NCOL; j += 4) {
        const int p = j / CPR, c = j - p * CPR;
        *reinterpret_cast<float4*>(sm.stage + p * 128 * CPR + ((c >> 2) * 128 + tid) * 4) =
            make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < NCOL; j += 2)
        *reinterpret_cast<float2*>(sm.stage + (j >> 1) * 256 + tid * 2) = make_float2(acc[j], acc[j + 1]);
    }
    fence_proxy_async_smem();
    cluster_sync();  // all stages written, every CTA's ring drained and receive barrier armed
    constexpr uint32_t slice_bytes = static_cast<uint32_t>(128 * CPR * 4);
    if (tid < S) {
      const uint32_t dst = cluster_map(smem_u32(sm.recv) + rank * slice_bytes, static_cast<uint32_t>(tid));
      const uint32_t bar = cluster_map(smem_u32(sm.xbar), static_cast<uint32_t>(tid));
      bulk_copy_to_peer(dst, smem_u32(sm.stage) + tid * slice_bytes, slice_bytes, bar);
    }
    if (!mbar_wait(sm.xbar, 0)) { record_error(a.status, DEV_TIMEOUT_EPI); sm.flags[0] = 1; }
    float v[CPR];
    dec_sum_slices<S, NCOL>(sm.recv, tid, v);
    // Every copy into this CTA has landed; once all CTAs pass the final barrier, every copy out of
    // this CTA's stage has too.
    cluster_arrive();
    __syncthreads();  // all slices summed before the epilogue reuses the receive buffer
    if (nvalid > 0 && sm.flags[0] == 0) {
      if constexpr (EPI == EPI_RESID) {
        const int n = m0 + tid;
        const float b = a.bias != nullptr ? a.bias[n] : 0.0f;
#pragma unroll
        for (int i = 0; i < CPR; ++i)
          if (i < nvalid)
            a.out_f32[static_cast<size_t>(c0 + i) * a.ld_out + n] = __fadd_rn(pre[i], __fadd_rn(out_round<RND>(v[i]), b));
      } else if constexpr (EPI == EPI_QKV) {
        dec_epilogue_qkv<CPR, RND>(a, v, c0, nvalid, m0, tid, sm.xs, pos0, pre, pre2);
      } else if constexpr (EPI == EPI_SWIGLU) {
        dec_epilogue_swiglu<CPR, RND>(a, v, c0, nvalid, m0, tid, sm.xs);
      } else {
        float vv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) vv[i] = i < CPR ? v[i < CPR ? i : 0] : 0.0f;
        gemm_epilogue_chunk_t<EPI, RND>(a, vv, c0, nvalid, m0, tid, sm.xs, pos0);
      }
    }
    cluster_wait();
  }
}

// One decode linear: CTA (m-tile, 1, split) of a grid whose z extent is the split-K factor S,
// launched as clusters of S CTAs along z. Instantiated per epilogue, split factor and weight format
// (bf16, or 4-bit affine with tmA over the packed nibbles) so that each kernel carries only the
// code it runs (the instruction cache is cold at every launch).
template <int EPI, int S, int QB>
__global__ void __launch_bounds__(128, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  constexpr bool QUANT = QB != 0;
  const int stages = QUANT ? kDecQStages : a.stages;
  const int kbs = a.kb_per_split;
  DecSmem sm;
  sm.ring = smem;
  sm.sB = smem + dec_ring_bytes(stages);
  sm.sP = sm.sB + static_cast<size_t>(kbs) * kDecBBytes;
  sm.qsc = reinterpret_cast<float*>(sm.sP + static_cast<size_t>(kbs) * dec_p_bytes(QB));
  sm.qbi = sm.qsc + kbs * 128;
  sm.stage = reinterpret_cast<float*>(smem);
  sm.recv = sm.stage + 128 * kDecRows;
  sm.xs = sm.recv;  // epilogue scratch, once the received slices are summed
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (QUANT ? dec_q_body_bytes(kbs, QB) : dec_body_bytes(stages, kbs)));
  sm.fullA = bars;
  sm.emptyA = bars + stages;
  sm.fullB = bars + 2 * stages;
  sm.accum = sm.fullB + 1;
  sm.xbar = sm.fullB + 2;
  sm.fullP = sm.fullB + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm.fullB + 4);
  sm.flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] error

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int m0 = blockIdx.x * 128;
  const int kb_total = a.K >> 6;
  const int kb0 = blockIdx.z * kbs;
  const int nkb = max(0, min(kbs, kb_total - kb0));

  if (tid == 0) {
    for (int st = 0; st < stages; ++st) {
      mbar_init(&sm.fullA[st], 1);
      mbar_init(&sm.emptyA[st], 1);
    }
    mbar_init(sm.fullB, 1);
    mbar_init(sm.accum, 1);
    mbar_init(sm.xbar, 1);
    mbar_init(sm.fullP, 1);
    sm.flags[0] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  // Weight prefetch first: it depends on nothing the producer kernel writes. At most
  // kDecPreStages K blocks: the activation tile, requested after the dependency wait, goes through
  // the same TMA unit and waits behind whatever is still being requested (Qwen3-0.6B decode step
  // at K/V length 4128: 1.53 ms with 2 blocks, 1.55 with 1, 1.54 with 3, 1.57 with the whole ring);
  // the producer requests the remaining blocks after it.
  const int npre = QUANT ? 0 : min(min(stages, nkb), kDecPreStages);
  uint64_t policy = 0;
  if (tid == 0) {
    policy = l2_policy_evict_first();
    if constexpr (QUANT) {
      if (nkb > 0) {
        mbar_expect_tx(sm.fullP, static_cast<uint32_t>(nkb * dec_p_bytes(QB)));
        for (int g = 0; g < nkb; ++g)
          tma_load_2d_hint(sm.sP + g * dec_p_bytes(QB), &tmA, sm.fullP, (kb0 + g) * (64 * QB / 8), m0, policy);
      }
    } else {
      for (int i = 0; i < npre; ++i) {
        mbar_expect_tx(&sm.fullA[i], kDecABytes);
        tma_load_2d_hint(sm.ring + static_cast<size_t>(i) * kDecABytes, &tmA, &sm.fullA[i], (kb0 + i) * 64, m0, policy);
      }
    }
  }
  if constexpr (QUANT) {
    // This thread's row: its scale and bias for every group of the K slice.
    const size_t base = static_cast<size_t>(m0 + tid) * a.q_groups + kb0;
    for (int g = 0; g < nkb; ++g) {
      sm.qsc[g * 128 + tid] = __bfloat162float(a.q_scale[base + g]);
      sm.qbi[g * 128 + tid] = __bfloat162float(a.q_bias[base + g]);
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
  // MMA width from the live row count, uniform across the cluster.
  if (rows_valid <= 32)
    dec_run<EPI, S, 32, QB>(&tmA, &tmB, a, sm, tmem, m0, kb0, nkb, npre, stages, policy, rows_valid, pos0);
  else
    dec_run<EPI, S, 64, QB>(&tmA, &tmB, a, sm, tmem, m0, kb0, nkb, npre, stages, policy, rows_valid, pos0);

  if (sm.flags[0] != 0 && tid == 0) {
    for (int st = 0; st < npre; ++st) mbar_wait(&sm.fullA[st], 0);
    if (QUANT && nkb > 0) mbar_wait(sm.fullP, 0);
    if (nkb > 0) mbar_wait(sm.fullB, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

// ---------------------------------------------------------------- lm_head over the decode rows
// The vocabulary projection of a decode step (n_out = V, e.g. 151936 = 1187 weight tiles, K = H)
// as one persistent CTA per SM that walks a contiguous run of weight tiles: the tiles of
// consecutive vocabulary rows are one contiguous range of HBM (128 rows x K x 2 bytes each), the
// activation tile is loaded once per CTA instead of once per weight tile, and the weight ring keeps
// streaming across tile boundaries. Warp-specialised (kLmThreads = 192): warps 0-3 read the f32
// accumulator (TMEM lane quarter = warp) and store the logits; warp 4 is the TMA producer, warp 5
// issues the UMMAs. The accumulator is double-buffered in TMEM (two blocks of 64 columns), so the
// MMAs of tile t + 1 run while the epilogue of tile t stores. Output: f32 logits rounded to bf16
// (the EPI_STORE_F32 epilogue of the other decode linears, same values). All waits are bounded.
constexpr int kLmThreads = 192;
constexpr int kLmMaxKb = 16;   // K <= 1024: the whole activation tile stays resident
__host__ __device__ inline size_t lm_smem_bytes(int stages, int nkb) {
  // alignment slack + B tile + ring + barriers (2 stages + fullB + 2 full + 2 empty + drain), TMEM
  // slot, flags
  return 1024 + static_cast<size_t>(nkb) * kDecBBytes + static_cast<size_t>(stages) * kDecABytes +
         static_cast<size_t>(2 * stages + 6) * 8 + 32;
}

template <int NCOL>
__device__ __forceinline__ void lm_run(const CUtensorMap* tmA, const CUtensorMap* tmB, const GemmArgs& a, uint8_t* sB,
                                       uint8_t* ring, uint64_t* fullA, uint64_t* emptyA, uint64_t* fullB, uint64_t* accF,
                                       uint64_t* accE, uint64_t* drain, volatile int* flags, uint32_t tmem, int tile0,
                                       int ntiles, int nkb, int stages, int rows_valid) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int total = ntiles * nkb;
  if (warp == 4) {
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      bool ok = true;
      // Weight K blocks continue from the ones requested before the dependency wait (kDecPreStages).
      int g = min(total, min(stages, kDecPreStages));
      for (; g < total; ++g) {
        const int s = g % stages;
        if (g >= stages && !mbar_wait(&emptyA[s], ((g / stages) - 1) & 1)) { ok = false; break; }
        if (flags[0] != 0) break;
        mbar_expect_tx(&fullA[s], kDecABytes);
        tma_load_2d_hint(ring + static_cast<size_t>(s) * kDecABytes, tmA, &fullA[s], (g % nkb) * 64, (tile0 + g / nkb) * 128,
                         policy);
      }
      flags[1] = g;  // weight K blocks requested
      if (!ok) { record_error(a.status, DEV_TIMEOUT_TMA); flags[0] = 1; }
    }
    __syncwarp();
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, NCOL);
      bool ok = total == 0 || mbar_wait(fullB, 0);
      int g = 0;
      for (int t = 0; t < ntiles && ok; ++t) {
        const int buf = t & 1;
        if (t >= 2 && !mbar_wait(&accE[buf], ((t >> 1) - 1) & 1)) { ok = false; break; }
        if (flags[0] != 0) { ok = false; break; }
        tc_fence_after();
        for (int i = 0; i < nkb; ++i, ++g) {
          const int s = g % stages;
          if (!mbar_wait(&fullA[s], (g / stages) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + static_cast<size_t>(s) * kDecABytes);
          const uint32_t b_addr = smem_u32(sB + static_cast<size_t>(i) * kDecBBytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + buf * 64, sdesc_kmajor_sw128(a_addr + kk * 32), sdesc_kmajor_sw128(b_addr + kk * 32), idesc,
                      (i | kk) != 0 ? 1u : 0u);
          umma_commit(&emptyA[s]);
        }
        if (ok) umma_commit(&accF[buf]);
      }
      flags[2] = g;  // weight K blocks whose bytes landed
      if (!ok) {
        record_error(a.status, DEV_TIMEOUT_MMA);
        flags[0] = 1;
      }
    }
    __syncwarp();
  } else {
    // Epilogue: thread tid holds vocabulary row m0 + tid of each tile.
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t & 1;
      // Both exits are decided per warp: the TMEM loads below are warp-collective.
      if (__any_sync(0xffffffffu, flags[0] != 0)) break;
      const bool ready = __all_sync(0xffffffffu, mbar_wait(&accF[buf], (t >> 1) & 1));
      if (!ready) {
        if (lane == 0) { record_error(a.status, DEV_TIMEOUT_EPI); flags[0] = 1; }
        break;
      }
      tc_fence_after();
      float acc[NCOL];
#pragma unroll
      for (int cb = 0; cb < NCOL; cb += 32) tmem_ld32(tmem + lane_off + buf * 64 + cb, acc + cb);
      tc_fence_before();
      mbar_arrive(&accE[buf]);  // this thread is done with the buffer: tile t + 2 may overwrite it
      const int m0 = (tile0 + t) * 128;
      gemm_epilogue_chunk_t<EPI_STORE_F32, true>(a, acc, 0, min(32, rows_valid), m0, tid, nullptr, 0);
      if constexpr (NCOL == 64)
        if (rows_valid > 32) gemm_epilogue_chunk_t<EPI_STORE_F32, true>(a, acc + 32, 32, rows_valid - 32, m0, tid, nullptr, 0);
    }
  }
}

__global__ void __launch_bounds__(kLmThreads, 1)
    gemm_lm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  const int stages = a.stages;
  const int nkb = a.K >> 6;
  uint8_t* sB = smem;
  uint8_t* ring = smem + static_cast<size_t>(nkb) * kDecBBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(stages) * kDecABytes);
  uint64_t* fullA = bars;
  uint64_t* emptyA = bars + stages;
  uint64_t* fullB = bars + 2 * stages;
  uint64_t* accF = fullB + 1;  // [2]
  uint64_t* accE = fullB + 3;  // [2]
  uint64_t* drain = fullB + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fullB + 6);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] error, [1] requested, [2] landed

  const int tid = threadIdx.x, warp = tid >> 5;
  // This CTA's run of consecutive weight tiles (the grid splits the tiles evenly, one CTA per SM).
  const int tiles_m = a.n_out >> 7;
  const int tile0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * tiles_m) / gridDim.x);
  const int ntiles = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * tiles_m) / gridDim.x) - tile0;
  const int total = ntiles * nkb;
  const int npre = min(total, min(stages, kDecPreStages));
  if (tid == 0) {
    for (int st = 0; st < stages; ++st) {
      mbar_init(&fullA[st], 1);
      mbar_init(&emptyA[st], 1);
    }
    mbar_init(fullB, 1);
    mbar_init(&accF[0], 1);
    mbar_init(&accF[1], 1);
    mbar_init(&accE[0], 128);
    mbar_init(&accE[1], 128);
    mbar_init(drain, 1);
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    // The first weight K blocks need nothing from the producer kernel.
    const uint64_t policy = l2_policy_evict_first();
    for (int g = 0; g < npre; ++g) {
      mbar_expect_tx(&fullA[g], kDecABytes);
      tma_load_2d_hint(ring + static_cast<size_t>(g) * kDecABytes, &tmA, &fullA[g], (g % nkb) * 64, (tile0 + g / nkb) * 128,
                       policy);
    }
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 128);
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
  if (tid == 0 && total > 0) {
    mbar_expect_tx(fullB, static_cast<uint32_t>(nkb * kDecBBytes));
    for (int i = 0; i < nkb; ++i) tma_load_2d(sB + static_cast<size_t>(i) * kDecBBytes, &tmB, fullB, i * 64, 0);
  }
  griddep_launch_dependents();
  if (rows_valid <= 32)
    lm_run<32>(&tmA, &tmB, a, sB, ring, fullA, emptyA, fullB, accF, accE, drain, flags, tmem, tile0, ntiles, nkb, stages,
               rows_valid);
  else
    lm_run<64>(&tmA, &tmB, a, sB, ring, fullA, emptyA, fullB, accF, accE, drain, flags, tmem, tile0, ntiles, nkb, stages,
               rows_valid);

  __syncthreads();
  if (flags[0] != 0 && warp == 5 && (tid & 31) == 0) {
    // A wait gave up (in whichever warp): every UMMA this thread issued completes before TMEM is
    // released, since the epilogue may have stopped reading while MMAs were still in flight.
    umma_commit(drain);
    mbar_wait(drain, 0);
  }
  if (flags[0] != 0 && tid == 0) {
    // A wait gave up: let every copy this CTA requested land before the shared memory goes away.
    // The producer runs at most `stages` blocks ahead of the last block whose bytes landed, so the
    // blocks in between occupy distinct slots and each is the newest request on its slot.
    if (total > 0) mbar_wait(fullB, 0);
    for (int g = flags[2]; g < flags[1]; ++g) mbar_wait(&fullA[g % stages], (g / stages) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

using DecGemmKernel = void (*)(const CUtensorMap, const CUtensorMap, const GemmArgs);

// The instantiation for an epilogue kind, split factor and weight format (qbits 0: bf16, 4: 4-bit
// affine, 8: int8 weight-only; nullptr if none).
inline DecGemmKernel dec_gemm_kernel(int epi, int S, int qbits = 0) {
#define DRT_DEC_ROW(E, Q)                                                                                              \
  {                                                                                                                    \
    gemm_decode_kernel<E, 1, Q>, gemm_decode_kernel<E, 2, Q>, gemm_decode_kernel<E, 4, Q>, gemm_decode_kernel<E, 8, Q>, \
        gemm_decode_kernel<E, 16, Q>                                                                                   \
  }
  static const DecGemmKernel table[3][4][5] = {
      {DRT_DEC_ROW(EPI_STORE_F32, 0), DRT_DEC_ROW(EPI_RESID, 0), DRT_DEC_ROW(EPI_SWIGLU, 0), DRT_DEC_ROW(EPI_QKV, 0)},
      {DRT_DEC_ROW(EPI_STORE_F32, 4), DRT_DEC_ROW(EPI_RESID, 4), DRT_DEC_ROW(EPI_SWIGLU, 4), DRT_DEC_ROW(EPI_QKV, 4)},
      {DRT_DEC_ROW(EPI_STORE_F32, 8), DRT_DEC_ROW(EPI_RESID, 8), DRT_DEC_ROW(EPI_SWIGLU, 8), DRT_DEC_ROW(EPI_QKV, 8)}};
#undef DRT_DEC_ROW
  const int si = S == 1 ? 0 : S == 2 ? 1 : S == 4 ? 2 : S == 8 ? 3 : S == 16 ? 4 : -1;
  const int qi = qbits == 0 ? 0 : qbits == 4 ? 1 : qbits == 8 ? 2 : -1;
  if (epi < 0 || epi > EPI_QKV || si < 0 || qi < 0) return nullptr;
  return table[qi][epi][si];
}

}  // namespace drt
