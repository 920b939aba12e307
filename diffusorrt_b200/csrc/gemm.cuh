// Skinny-M linear layers on the 5th-generation tensor cores.
//
// Every linear in the decode step is y = x @ W^T with W [n_out, K] bf16 and x [rows, K] bf16
// (rows = 32..64 active canvas rows per denoising step, up to thousands for a prompt
// prefill). The kernel computes the transposed product D^T = W . x^T so the weight tile is
// the M = 128 operand of tcgen05.mma and the activation rows are the N operand (N = BN); the
// f32 accumulator lives in TMEM with weight row m in TMEM lane m and activation row n in
// column n. Weights stream from HBM through a TMA ring (SWIZZLE_128B, evict-first hint); the
// activation tile for the same K block arrives on its own barrier so that, under
// programmatic dependent launch, the weight prefetch of this kernel overlaps the tail of the
// kernel that produces x. Warp 0 issues TMA, warp 1 issues UMMA, all four warps run the epilogue.
//
// Split-K: grid.z CTAs share one output tile and form one thread-block cluster. Each pushes
// column slice r of its f32 partial into CTA r's shared memory (remote stores), and after the
// cluster barrier CTA r sums its slice over all partials in rank order and runs the epilogue for
// those columns. No global workspace, no atomics, and results do not depend on scheduling.
//
// Epilogues follow the MLX precision contract of the reference forward
// (python/src/edllm/backends/mlx_ops.py:97-130 linear, :21-35 rms_norm, :133-144 rope,
// :147-154 swiglu): the bf16 x bf16 matmul output is rounded to bf16 and widened to f32,
// bias is added in f32, and the residual stream stays f32.
#pragma once
#include "common.cuh"

namespace drt {

enum GemmEpilogue : int {
  EPI_STORE_F32 = 0,  // out_f32[row, n] = bf16r(acc) + bias        (logits, tests)
  EPI_RESID = 1,      // out_f32[row, n] += bf16r(acc) + bias       (o_proj / down_proj)
  EPI_SWIGLU = 2,     // out_bf16[row, j] = bf16(silu(g) * u)       (gate/up interleaved per tile)
  EPI_QKV = 3,        // q/k RMSNorm + RoPE; q -> q buffer, k -> K cache, v -> V^T cache
  EPI_STORE_RAW = 4,  // out_f32[row, n] = acc (no rounding; tests)
  EPI_TP_PUSH = 5,    // tensor parallel: acc (f32) into this rank's slot of the receive buffer of
                      // the rank owning the tile's features (NVLink peer store when that is another
                      // GPU); the last CTA raises this rank's flag on every rank
  EPI_TP_GATHER = 6,  // vocabulary-parallel lm_head: bf16r(acc) + bias into every rank's logits
                      // (tp_dst[r] already offset to this rank's first vocabulary column); the last
                      // CTA raises this rank's flag on every rank
};

constexpr int kTpMaxRanks = 8;

struct GemmArgs {
  int n_out;             // rows of W; multiple of 128
  int K;                 // multiple of 64
  int rows;              // activation rows covered by the grid
  const int* rows_dev;   // optional device-side row count (<= rows) for static graphs
  int splits;            // split-K factor = cluster size along z (1, 2, 4, 8 or 16)
  int kb_per_split;      // K blocks of 64 per split (the last split takes the remainder)
  int stages;            // smem ring depth
  int* status;           // device error word
  int epi;
  // epilogue operands
  float* out_f32;
  __nv_bfloat16* out_bf16;
  int ld_out;            // row stride (elements) of out_f32 / out_bf16
  const float* bias;     // optional [n_out] (f32 copy of the bf16 bias)
  // EPI_QKV
  const float* qnorm_w;  // [128] or null (no QK-norm)
  const float* knorm_w;  // [128] or null
  const float* rope_cos; // [max_pos][64]
  const float* rope_sin; // [max_pos][64]
  int pos0;              // absolute position of activation row 0
  const int* pos0_dev;   // optional device-side pos0
  int nq, nkv;
  __nv_bfloat16* kcache; // this layer: [nkv][max_seq][128]
  __nv_bfloat16* vtcache;// this layer: [nkv][128][max_seq]
  int max_seq;
  float eps;
  // stream-K (gemm_streamk_kernel): per-CTA partial tiles [grid][BN][128] f32 and ready flags [grid]
  float* sk_part;
  int* sk_flag;
  // 4-bit affine weights (decode linear, quantized instantiation): per (row, group of 64 inputs)
  // bf16 scale and bias, [n_out][q_groups] with q_groups = K / 64; the packed nibbles come from tmA.
  const __nv_bfloat16* q_scale;
  const __nv_bfloat16* q_bias;
  int q_groups;
  // EPI_TP_PUSH: per rank r, this rank's slot of r's receive buffer ([rows][ld_out] f32) and this
  // rank's flag in r's flag array; a local arrival counter; the forward's epoch and this linear's tag
  // (the flag value is tp_flag_value(epoch, tag)). Feature tile t (128 features) is owned by rank t % world.
  float* tp_dst[kTpMaxRanks];
  unsigned long long* tp_flag[kTpMaxRanks];
  int* tp_count;
  const unsigned long long* tp_epoch;
  int tp_world, tp_tag;
  int tp_all;  // store to every rank instead of the owner only
};

// KS: K blocks of 64 per ring stage. One mbarrier phase covers a whole stage; larger stages keep
// more bytes in flight per barrier round trip, which is what bounds one CTA's TMA ingest rate.
template <int BN, int KS = 1>
struct GemmCfg {
  static constexpr int kABytes = 128 * 128;       // 128 rows x 64 bf16 (one K block)
  static constexpr int kBBytes = BN * 128;        // BN rows x 64 bf16 (one K block)
  static constexpr int kStageBytes = KS * (kABytes + kBBytes);
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  // Ring, or (split-K, BN <= 128) the receive buffer plus the epilogue exchange buffer, whichever is
  // larger. Wider tiles are never split and only need the exchange buffer after the ring drains.
  __host__ __device__ static size_t body_bytes(int stages) {
    const size_t ring = static_cast<size_t>(stages) * kStageBytes;
    const size_t recv = BN <= 128 ? static_cast<size_t>(BN) * 128 * 4 : 0;
    const size_t epi = recv + (32 * 128 + 160) * 4;
    return ((ring > epi ? ring : epi) + 1023) & ~size_t(1023);
  }
  __host__ __device__ static size_t smem_bytes(int stages) { return 1024 + body_bytes(stages) + 256; }
};

// Linear output rounding: the bf16-weight contract rounds the matmul output to bf16
// (mlx_ops.py:122-125); the quantized-weight contract (mx.quantized_matmul, mlx_ops.py:108-117)
// keeps the f32 result.
template <bool RND>
__device__ __forceinline__ float out_round(float x) {
  if constexpr (RND) return bf16_round(x);
  else return x;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Epilogue for up to 32 accumulator columns (activation rows col0 .. col0+ncols-1).
// v[i] holds this thread's weight row (m0 + tid) for activation row col0 + i. All loops run to
// 32 with a guard so v stays in registers.
// xs: shared scratch of at least 32 x 132 floats (SwiGLU, QKV).
template <int EPI, bool RND = true>
__device__ __forceinline__ void gemm_epilogue_chunk_t(const GemmArgs& a, float* v, int col0, int ncols, int m0, int tid,
                                                      float* xs, int pos0) {
  const int n = m0 + tid;
  const float b = a.bias != nullptr ? a.bias[n] : 0.0f;
    if constexpr (EPI == EPI_STORE_RAW) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < ncols) a.out_f32[static_cast<size_t>(col0 + i) * a.ld_out + n] = v[i];
    }
    if constexpr (EPI == EPI_TP_PUSH) {
      // to the owning rank (reduce-scatter), or to every rank when tp_all (each rank reduces all)
      const int owner = (m0 >> 7) % a.tp_world;
      for (int r = a.tp_all ? 0 : owner; r < (a.tp_all ? a.tp_world : owner + 1); ++r) {
        float* dst = a.tp_dst[r];
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < ncols) dst[static_cast<size_t>(col0 + i) * a.ld_out + n] = v[i];
      }
    }
    if constexpr (EPI == EPI_STORE_F32) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < ncols) a.out_f32[static_cast<size_t>(col0 + i) * a.ld_out + n] = __fadd_rn(out_round<RND>(v[i]), b);
    }
    if constexpr (EPI == EPI_TP_GATHER) {
      // the single-GPU head's values (EPI_STORE_F32), stored into every rank's logits
      float o[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = __fadd_rn(out_round<RND>(v[i]), b);
      for (int r = 0; r < a.tp_world; ++r) {
        float* dst = a.tp_dst[r];
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < ncols) dst[static_cast<size_t>(col0 + i) * a.ld_out + n] = o[i];
      }
    }
    if constexpr (EPI == EPI_RESID) {
      float cur[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) cur[i] = i < ncols ? a.out_f32[static_cast<size_t>(col0 + i) * a.ld_out + n] : 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        cur[i] = __fadd_rn(cur[i], __fadd_rn(out_round<RND>(v[i]), b));
        if (i < ncols) a.out_f32[static_cast<size_t>(col0 + i) * a.ld_out + n] = cur[i];
      }
    }
    if constexpr (EPI == EPI_SWIGLU) {
      // Tile layout (set by the weight packer): lanes 0..63 = gate rows j0..j0+63,
      // lanes 64..127 = up rows j0..j0+63 of the same intermediate features.
      // All four warps: every lane parks its 32 values, then lane pair (f, f + 64) splits the rows by
      // parity, so each thread evaluates 16 SwiGLU outputs instead of half the threads 32.
      const int j0 = (m0 >> 1);
#pragma unroll
      for (int i = 0; i < 32; ++i) xs[i * 128 + tid] = __fadd_rn(out_round<RND>(v[i]), b);
      __syncthreads();
      const int f = tid & 63, par = tid >> 6;
      float g[16], u[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        g[k] = xs[(2 * k + par) * 128 + f];
        u[k] = xs[(2 * k + par) * 128 + 64 + f];
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int i = 2 * k + par;
        if (i < ncols) {
          const float sig = 1.0f / (1.0f + expf(-g[k]));
          const float act = __fmul_rn(__fmul_rn(g[k], sig), u[k]);
          a.out_bf16[static_cast<size_t>(col0 + i) * a.ld_out + j0 + f] = __float2bfloat16_rn(act);
        }
      }
      __syncthreads();
    }
    if constexpr (EPI == EPI_QKV) {
      const int tile = m0 >> 7;
      const bool is_q = tile < a.nq;
      const bool is_k = !is_q && tile < a.nq + a.nkv;
      if (!is_q && !is_k) {
        // V: no norm, no rope. Written transposed: V^T[g][d][pos], contiguous along pos.
        const int g = tile - a.nq - a.nkv;
        __nv_bfloat16* dst = a.vtcache + (static_cast<size_t>(g) * 128 + tid) * a.max_seq + pos0 + col0;
        const bool vec = (ncols == 32) && (((pos0 + col0) & 7) == 0);
        if (vec) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            __align__(16) __nv_bfloat16 t[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) t[e] = __float2bfloat16_rn(__fadd_rn(out_round<RND>(v[q * 8 + e]), b));
            *reinterpret_cast<uint4*>(dst + q * 8) = *reinterpret_cast<const uint4*>(t);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < ncols) dst[i] = __float2bfloat16_rn(__fadd_rn(out_round<RND>(v[i]), b));
        }
        return;
      }
      const float* nw = is_q ? a.qnorm_w : a.knorm_w;
      // The chunk is staged in shared memory and re-read with four threads per row: thread t owns
      // row i = t / 4 and features [16 q, 16 q + 16) and [64 + 16 q, 80 + 16 q), q = t % 4, so the
      // RoPE partners (f, f + 64) sit in the same thread, the row's sum of squares takes two
      // shuffles (no block barrier), and every store is a 32-byte run of the row.
      constexpr int kLd = 132;  // padded row stride (floats) of the staged chunk
#pragma unroll
      for (int i = 0; i < 32; ++i) xs[i * kLd + tid] = __fadd_rn(out_round<RND>(v[i]), b);
      __syncthreads();
      const int i = tid >> 2, q = tid & 3;
      const int f0 = q * 16;
      float lo[16], hi[16];
#pragma unroll
      for (int e = 0; e < 16; e += 4) {
        const float4 l4 = *reinterpret_cast<const float4*>(xs + i * kLd + f0 + e);
        const float4 h4 = *reinterpret_cast<const float4*>(xs + i * kLd + 64 + f0 + e);
        lo[e] = l4.x; lo[e + 1] = l4.y; lo[e + 2] = l4.z; lo[e + 3] = l4.w;
        hi[e] = h4.x; hi[e + 1] = h4.y; hi[e + 2] = h4.z; hi[e + 3] = h4.w;
      }
      __syncthreads();  // the staged chunk is consumed; the caller may stage the next one
      const int pos = pos0 + col0 + max(0, min(i, ncols - 1));
      if (nw != nullptr) {
        float ss = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) ss = __fmaf_rn(lo[e], lo[e], ss);
#pragma unroll
        for (int e = 0; e < 16; ++e) ss = __fmaf_rn(hi[e], hi[e], ss);
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), a.eps)));
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          lo[e] = __fmul_rn(__fmul_rn(lo[e], rs), __ldg(nw + f0 + e));
          hi[e] = __fmul_rn(__fmul_rn(hi[e], rs), __ldg(nw + 64 + f0 + e));
        }
      }
      // RoPE: (x_f, x_{f+64}) -> (x_f c - x_{f+64} s, x_{f+64} c + x_f s), c / s of (pos, f)
      const float* cp = a.rope_cos + static_cast<size_t>(pos) * 64 + f0;
      const float* sp = a.rope_sin + static_cast<size_t>(pos) * 64 + f0;
      __align__(16) __nv_bfloat16 olo[16], ohi[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float c = __ldg(cp + e), sn = __ldg(sp + e);
        olo[e] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(lo[e], c), __fmul_rn(-hi[e], sn)));
        ohi[e] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(hi[e], c), __fmul_rn(lo[e], sn)));
      }
      if (i < ncols) {
        const int head = is_q ? tile : tile - a.nq;
        __nv_bfloat16* dst = is_q ? a.out_bf16 + (static_cast<size_t>(col0 + i) * a.nq + head) * 128
                                  : a.kcache + (static_cast<size_t>(head) * a.max_seq + pos) * 128;
        *reinterpret_cast<uint4*>(dst + f0) = *reinterpret_cast<const uint4*>(olo);
        *reinterpret_cast<uint4*>(dst + f0 + 8) = *reinterpret_cast<const uint4*>(olo + 8);
        *reinterpret_cast<uint4*>(dst + 64 + f0) = *reinterpret_cast<const uint4*>(ohi);
        *reinterpret_cast<uint4*>(dst + 64 + f0 + 8) = *reinterpret_cast<const uint4*>(ohi + 8);
      }
    }
}

// Runtime dispatch over the epilogue kinds (the prefill kernel, whose epilogue is a launch argument).
__device__ __forceinline__ void gemm_epilogue_chunk(const GemmArgs& a, float* v, int col0, int ncols, int m0, int tid,
                                                    float* xs, int pos0) {
  switch (a.epi) {
    case EPI_STORE_RAW: gemm_epilogue_chunk_t<EPI_STORE_RAW>(a, v, col0, ncols, m0, tid, xs, pos0); break;
    case EPI_STORE_F32: gemm_epilogue_chunk_t<EPI_STORE_F32>(a, v, col0, ncols, m0, tid, xs, pos0); break;
    case EPI_RESID: gemm_epilogue_chunk_t<EPI_RESID>(a, v, col0, ncols, m0, tid, xs, pos0); break;
    case EPI_SWIGLU: gemm_epilogue_chunk_t<EPI_SWIGLU>(a, v, col0, ncols, m0, tid, xs, pos0); break;
    case EPI_QKV: gemm_epilogue_chunk_t<EPI_QKV>(a, v, col0, ncols, m0, tid, xs, pos0); break;
    case EPI_TP_PUSH: gemm_epilogue_chunk_t<EPI_TP_PUSH>(a, v, col0, ncols, m0, tid, xs, pos0); break;
    case EPI_TP_GATHER: gemm_epilogue_chunk_t<EPI_TP_GATHER>(a, v, col0, ncols, m0, tid, xs, pos0); break;
    default: break;
  }
}

// Split-K exchange inside one cluster of S CTAs. Each thread holds its weight row's f32 partial
// for all BN activation rows; column slice j (BN / S columns) belongs to CTA j. Every thread
// pushes slice j into CTA j's receive buffer recv[src rank][thread][BN / S] with remote
// shared-memory stores; after the cluster barrier each CTA sums its own slice over the S sources
// in rank order from local shared memory.
template <int BN, int S>
__device__ __forceinline__ void split_push(const float* acc, float* recv, uint32_t rank, int tid) {
  constexpr int CPR = BN / S;
  constexpr int QP = CPR / 4;
  static_assert(CPR >= 4 && CPR <= 32, "split slice must be 4..32 columns");
  const uint32_t base = smem_u32(recv) + static_cast<uint32_t>(((rank * 128 + tid) * CPR) * 4);
#pragma unroll
  for (int j = 0; j < S; ++j) {
    const uint32_t dst = cluster_map(base, static_cast<uint32_t>(j));
#pragma unroll
    for (int q = 0; q < QP; ++q) {
      const int c = j * CPR + q * 4;
      st_cluster_f32x4(dst + q * 16, make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]));
    }
  }
}

template <int BN, int S>
__device__ __forceinline__ int split_sum(const float* recv, uint32_t rank, int tid, float* v, int* c0_out) {
  constexpr int CPR = BN / S;
  constexpr int QP = CPR / 4;
#pragma unroll
  for (int q = 0; q < QP; ++q) {
    float4 acc = *reinterpret_cast<const float4*>(recv + tid * CPR + q * 4);
#pragma unroll
    for (int p = 1; p < S; ++p) {
      const float4 t = *reinterpret_cast<const float4*>(recv + (p * 128 + tid) * CPR + q * 4);
      acc.x += t.x;
      acc.y += t.y;
      acc.z += t.z;
      acc.w += t.w;
    }
    v[4 * q] = acc.x;
    v[4 * q + 1] = acc.y;
    v[4 * q + 2] = acc.z;
    v[4 * q + 3] = acc.w;
  }
  *c0_out = static_cast<int>(rank) * CPR;
  return CPR;
}

template <int BN, int KS = 1>
__global__ void __launch_bounds__(128, 1)
    gemm_swapab_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const GemmArgs a) {
  using Cfg = GemmCfg<BN, KS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  const int stages = a.stages;
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + Cfg::body_bytes(stages));
  uint64_t* full = bars;               // A and B of a stage
  uint64_t* empty = bars + stages;
  uint64_t* accum = bars + 2 * stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] error

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // Tile order: with several row tiles, the CTAs that share a weight tile are consecutive in launch
  // order (row tile fastest), so the weight tile comes from HBM once and from L2 for the others.
  const int tiles_n = gridDim.y;
  const int bid = blockIdx.y * gridDim.x + blockIdx.x;
  const int m0 = (tiles_n > 1 ? bid / tiles_n : static_cast<int>(blockIdx.x)) * 128;
  const int n0 = (tiles_n > 1 ? bid % tiles_n : static_cast<int>(blockIdx.y)) * BN;
  const int split = blockIdx.z;
  const int kb_total = a.K >> 6;
  const int kb0 = split * a.kb_per_split;
  const int nkb = max(0, min(a.kb_per_split, kb_total - kb0));
  const int nsb = (nkb + KS - 1) / KS;  // ring stages to fill

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    flags[0] = 0;
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

  // Stage layout: KS weight tiles (A), then KS activation tiles (B). The stage's barrier is armed
  // once with every byte of the stage; the weight loads need nothing from the producer kernel, so
  // the first stages' weights are requested before the PDL wait and their activations after it.
  const int npre = min(stages, nsb);
  uint64_t policy = 0;
  if (tid == 0) {
    policy = tiles_n > 1 ? l2_policy_evict_normal() : l2_policy_evict_first();
    for (int i = 0; i < npre; ++i) {
      const int nk = min(KS, nkb - i * KS);
      uint8_t* st = ring + static_cast<size_t>(i) * Cfg::kStageBytes;
      mbar_expect_tx(&full[i], static_cast<uint32_t>(nk * (Cfg::kABytes + Cfg::kBBytes)));
      for (int j = 0; j < nk; ++j)
        tma_load_2d_hint(st + j * Cfg::kABytes, &tmA, &full[i], (kb0 + i * KS + j) * 64, m0, policy);
    }
  }
  griddep_wait();
  griddep_launch_dependents();

  // Warp 0: TMA producer. Warp 1: UMMA issuer. One elected lane each; the rest of the warp waits
  // at the warp barrier instead of spinning beside it.
  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < nsb && ok; ++i) {
        const int s = i % stages;
        const int nk = min(KS, nkb - i * KS);
        uint8_t* st = ring + static_cast<size_t>(s) * Cfg::kStageBytes;
        if (i >= stages) {
          if (!mbar_wait(&empty[s], ((i / stages) - 1) & 1)) { ok = false; break; }
          mbar_expect_tx(&full[s], static_cast<uint32_t>(nk * (Cfg::kABytes + Cfg::kBBytes)));
          for (int j = 0; j < nk; ++j)
            tma_load_2d_hint(st + j * Cfg::kABytes, &tmA, &full[s], (kb0 + i * KS + j) * 64, m0, policy);
        }
        for (int j = 0; j < nk; ++j)
          tma_load_2d(st + KS * Cfg::kABytes + j * Cfg::kBBytes, &tmB, &full[s], (kb0 + i * KS + j) * 64, n0);
      }
      if (!ok) { record_error(a.status, DEV_TIMEOUT_TMA); flags[0] = 1; }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, BN);
      bool ok = true;
      for (int i = 0; i < nsb; ++i) {
        const int s = i % stages;
        const int nk = min(KS, nkb - i * KS);
        const uint32_t ph = (i / stages) & 1;
        if (!mbar_wait(&full[s], ph)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(ring + static_cast<size_t>(s) * Cfg::kStageBytes);
        const uint32_t b_addr = a_addr + KS * Cfg::kABytes;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          if (j < nk) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              umma_bf16(tmem, sdesc_kmajor_sw128(a_addr + j * Cfg::kABytes + kk * 32),
                        sdesc_kmajor_sw128(b_addr + j * Cfg::kBBytes + kk * 32), idesc, (i | j | kk) != 0 ? 1u : 0u);
            }
          }
        }
        umma_commit(&empty[s]);
      }
      if (!ok) { record_error(a.status, DEV_TIMEOUT_MMA); flags[0] = 1; }
      umma_commit(accum);
    }
    __syncwarp();
  }

  // ---------------- epilogue (all four warps; warp w owns TMEM lanes [32w, 32w+32))
  bool acc_ok = true;
  if (nkb > 0) acc_ok = mbar_wait(accum, 0);
  tc_fence_after();
  if (!acc_ok) { record_error(a.status, DEV_TIMEOUT_EPI); flags[0] = 1; }
  __syncthreads();
  const bool failed = flags[0] != 0;
  int rows_valid = a.rows;
  if (a.rows_dev != nullptr) rows_valid = min(rows_valid, *a.rows_dev);
  const int pos0 = a.pos0_dev != nullptr ? *a.pos0_dev : a.pos0;
  const int ncol_valid = max(0, min(BN, rows_valid - n0));
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);

  if (a.splits == 1) {
    float* xs = reinterpret_cast<float*>(ring);  // exchange buffer over the drained ring
    if (!failed) {
      for (int cb = 0; cb < ncol_valid; cb += 32) {
        float v[32];
        tmem_ld32(lane_addr + cb, v);
        gemm_epilogue_chunk(a, v, n0 + cb, min(32, ncol_valid - cb), m0, tid, xs, pos0);
      }
    }
    if (a.epi == EPI_TP_PUSH || a.epi == EPI_TP_GATHER) {
      // Every CTA's peer stores are made visible system-wide before it arrives; the last CTA of the
      // grid then raises this rank's flag in every rank's flag array (failed CTAs arrive too, so
      // the peers' waits end; the status word carries the failure).
      __threadfence_system();
      __syncthreads();
      if (tid == 0) {
        const int total = static_cast<int>(gridDim.x * gridDim.y * gridDim.z);
        if (atomicAdd(a.tp_count, 1) + 1 == total) {
          __threadfence_system();
          const unsigned long long e =
              tp_flag_value(*reinterpret_cast<const volatile unsigned long long*>(a.tp_epoch), a.tp_tag);
          for (int r = 0; r < a.tp_world; ++r) st_release_sys(a.tp_flag[r], e);
          *a.tp_count = 0;
        }
      }
    }
  } else {
    // Split-K across the CTAs of one cluster (cluster dims 1 x 1 x splits). The receive buffer
    // overlays the ring, which a peer's pushes may only reach once this CTA's own UMMAs are done:
    // arrive here (own accumulator final), wait before pushing (every peer's accumulator final).
    cluster_arrive();
    float* recv = reinterpret_cast<float*>(ring);  // [splits][128][BN / splits]
    float* xs = recv + 128 * BN;
    const uint32_t rank = cluster_ctarank();
    float v[32];
    int c0 = 0, nc = 0;
    if constexpr (BN == 64) {
      float acc[BN];
      if (!failed && nkb > 0) {
#pragma unroll
        for (int cb = 0; cb < BN; cb += 32) tmem_ld32(lane_addr + cb, acc + cb);
      } else {
#pragma unroll
        for (int c = 0; c < BN; ++c) acc[c] = 0.0f;
      }
      cluster_wait();
      switch (a.splits) {
        case 2: split_push<BN, 2>(acc, recv, rank, tid); break;
        case 4: split_push<BN, 4>(acc, recv, rank, tid); break;
        case 8: split_push<BN, 8>(acc, recv, rank, tid); break;
        default: split_push<BN, 16>(acc, recv, rank, tid); break;
      }
      cluster_sync();
      switch (a.splits) {
        case 2: nc = split_sum<BN, 2>(recv, rank, tid, v, &c0); break;
        case 4: nc = split_sum<BN, 4>(recv, rank, tid, v, &c0); break;
        case 8: nc = split_sum<BN, 8>(recv, rank, tid, v, &c0); break;
        default: nc = split_sum<BN, 16>(recv, rank, tid, v, &c0); break;
      }
    } else {
      // Wider tiles (prompt prefill) are never split.
      cluster_wait();
      cluster_sync();
      if (tid == 0) record_error(a.status, DEV_BAD_SHAPE);
    }
    nc = max(0, min(nc, ncol_valid - c0));
    if (nc > 0 && !failed) gemm_epilogue_chunk(a, v, n0 + c0, nc, m0, tid, xs, pos0);
  }
  if (failed && tid == 0) {
    // Drain loads that may still be landing in this CTA's shared memory (bounded).
    for (int s = 0; s < min(stages, nsb); ++s) mbar_wait(&full[s], 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

}  // namespace drt
