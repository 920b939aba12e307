// Fused unmask selector: per-row vocabulary softmax statistics in float64, confidence and
// committed token, in one pass over HBM for max-prob and two for entropy.
//
// Max-prob (TopConfidence, python/src/edllm/backends/diffusion_runtime.py:179-192):
//   p = exp(f64(x) - max) / sum(exp(f64(x) - max)); conf = max p = 1 / S; token = argmax p.
//   exp is monotone and 1/S scales every entry equally, so argmax p is the FIRST index of the
//   largest f32 logit (integer-exact), and conf = 1 / S with S accumulated in f64.
// Entropy (NegEntropy, diffusion_runtime.py:90-114 without top-p):
//   a = f64(x) / T (T > 0), p = softmax(a), conf = f32(sum p * log(p + 1e-10)), token = argmax p.
//   With m = max a, e = exp(a - m), S = sum e and eps = 1e-10, log(p + eps) = log p + log1p(eps / p)
//   and log p = (a - m) - log S, so the sum splits into
//     H = (sum e (a - m)) / S - log S  +  C,   C = sum p log1p(eps / p).
//   The first part comes out of pass 1 in float64 (one more FMA per logit beside the sum of e;
//   every term has the same sign, so nothing cancels). 0 <= p log1p(eps / p) <= eps for every p,
//   so C <= V eps (1.5e-5 at V = 151936), about 15 float32 ulps of a typical |H|: pass 2 evaluates
//   each term of C / eps in float32 (relative error about 1e-6) and sums in float64, which puts H
//   within about 1e-13 of the float64 per-logit sum, far inside the half ulp the float32 cast keeps.
//
// Layout: grid (chunks, rows); each CTA reduces one chunk of a row to (max, first argmax,
// sum exp(x - chunk_max)); the last CTA of a row (arrival counter, reset by that CTA) merges
// the row's chunk partials in chunk order, so the result is independent of scheduling.
// S differs from NumPy's pairwise sum of its own exp in the last bits; the decode policy
// flags ranking decisions closer than the certified bound (see policy.cuh).
#pragma once
#include "common.cuh"
#include "fastexp.cuh"

namespace drt {

enum SelMode : int { SEL_MAXPROB = 0, SEL_ENTROPY = 1, SEL_SAMPLE = 2 };

// Temperature sampling for the fixed-quota policies (TopConfidence at T > 0, sampling_noise and
// _sampled_max_prob_confidence, python/src/edllm/backends/diffusion_runtime.py:195-253): row r's
// token is the first argmax of f64(x) + T * f64(g) (product and sum rounded separately), with the
// float32 Gumbel noise g = -log(-log u) and u = (top 23 bits + 1/2) * 2^-23 of a splitmix64 hash of
// (seed, forward index, canvas position, token); the row's confidence is the raw softmax
// probability of that token, exp(x_tok - max) / S. The float32 logs are CUDA's logf, which can
// differ from the host's in the last bit; that moves a draw only when two keys are within
// kSampleTieScale * T of each other, and such rows get DRT_TIE_NEAR.
constexpr unsigned long long kSampleGolden = 0x9E3779B97F4A7C15ull;
// |g| <= 17 for every u this hash can produce, and one last-bit difference in each f32 log moves g by
// at most 2^-21 (1 + |g|) < 2^-16: keys closer than 2^-16 T are not certified.
constexpr double kSampleTieScale = 1.52587890625e-05;  // 2^-16

// splitmix64's output function (Steele, Lea and Flood 2014).
__device__ __forceinline__ unsigned long long splitmix_mix(unsigned long long z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// Key of one (seed, forward, position) row: three chained mixes, each adding a golden-ratio step.
__device__ __forceinline__ unsigned long long sample_row_key(unsigned long long seed, int forward, int position) {
  unsigned long long k = splitmix_mix(seed + kSampleGolden);
  k = splitmix_mix(k + static_cast<unsigned long long>(forward + 1) * kSampleGolden);
  return splitmix_mix(k + static_cast<unsigned long long>(position + 1) * kSampleGolden);
}
__device__ __forceinline__ float sample_gumbel(unsigned long long row_key, int token) {
  const unsigned long long bits = splitmix_mix(row_key + static_cast<unsigned long long>(token + 1) * kSampleGolden);
  const float u = (static_cast<float>(bits >> 41) + 0.5f) * 1.1920928955078125e-07f;  // 2^-23, exact
  return -logf(-logf(u));
}
// Best key (lowest index among equals) and the runner-up value, merged in a fixed order.
__device__ __forceinline__ void top2_merge(double& b1, int& i1, double& b2, double v1, int j1, double v2) {
  if (v1 > b1 || (v1 == b1 && j1 < i1)) {
    b2 = fmax(b1, v2);
    b1 = v1;
    i1 = j1;
  } else {
    b2 = fmax(b2, v1);
  }
}

struct SelArgs {
  const float* logits;
  int64_t ld;             // row stride in floats
  const int* row_index;   // optional: row r reads logits row row_index[r]
  int rows;
  const int* rows_dev;    // optional device-side row count
  int vocab;
  int chunk;              // elements per CTA (kSelChunk)
  int nchunks;
  int mode;
  double temperature;     // entropy only; <= 0 means no scaling
  int exclude;            // token index scored as -inf (MASK exclusion), -1 for none
  const int* exclude_dev; // optional device-side override of `exclude`
  float* part_max;        // [rows * nchunks]
  int* part_idx;
  double* part_sum;
  double* part_ent;       // entropy: [rows * nchunks] sum e (a - chunk max) per chunk; slot 0 of a row
                          // then holds the row's sum e (a - m) / S - log S
  int* counters;          // [rows]
  double* row_amax;       // [rows] entropy: the row's largest float32 logit
  double* row_sum;        // [rows] S (entropy)
  double* conf;           // [rows]
  int* token;             // [rows]
  int* status;
  // SEL_SAMPLE, or SEL_MAXPROB with *sample_t_dev > 0: the Gumbel draw (see above)
  double sample_t;              // temperature (mode SEL_SAMPLE)
  const double* sample_t_dev;   // optional device-side temperature (a graph replays either mode)
  unsigned long long sample_seed;
  const unsigned long long* sample_seed_dev;
  int sample_forward;           // forward index keying the draw
  const int* sample_forward_dev;
  const int* positions;         // [rows] canvas position of each row
  double* part_skey;            // [rows * nchunks] best sampled key of each chunk
  double* part_skey2;           // runner-up key
  int* part_sidx;               // index of the best key
  int* row_tie;                 // optional [rows]: DRT_TIE_NEAR when the sampled argmax is not certified
};

constexpr int kSelThreads = 256;
constexpr int TIE_NEAR_BIT = 1;  // DRT_TIE_NEAR
constexpr int kSelChunk = 8192;  // logits per CTA: 32 per thread

__device__ __forceinline__ void argmax_merge(float& m, int& idx, float m2, int idx2) {
  if (m2 > m || (m2 == m && idx2 < idx)) {
    m = m2;
    idx = idx2;
  }
}

// x / T evaluated as x * (1 / T) (1 / T = 1 when T <= 0: no scaling); the product differs from the
// quotient in the last f64 bit at most and is exact for T = 1.
__device__ __forceinline__ double sel_inv_t(double T) { return T > 0.0 ? 1.0 / T : 1.0; }
__device__ __forceinline__ double sel_adjust(double x, double inv_t) { return x * inv_t; }

// Pass 1: chunk max / argmax / sum of exp relative to the chunk's adjusted max. kSample adds the
// sampled draw (SEL_SAMPLE, or SEL_MAXPROB with a device-side temperature above 0); the greedy
// instantiation carries none of its registers (64 -> 48 per thread, 4 -> 5 resident CTAs per SM).
// kEntropy (SEL_ENTROPY) also accumulates sum e (a - chunk max) for the entropy's exact part.
template <bool kSample, bool kEntropy = false>
__global__ void __launch_bounds__(kSelThreads, kSample ? 4 : 5) sel_pass1_kernel(const SelArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  int rows_valid = a.rows;
  if (a.rows_dev != nullptr) rows_valid = min(rows_valid, *a.rows_dev);
  const int r = blockIdx.y;
  if (r >= rows_valid) return;
  const int c = blockIdx.x;
  const int src = a.row_index != nullptr ? a.row_index[r] : r;
  const float* x = a.logits + static_cast<int64_t>(src) * a.ld;
  const int lo = c * a.chunk;
  const int hi = min(a.vocab, lo + a.chunk);
  const int tid = threadIdx.x;
  const bool vec = ((a.ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0);
  const int excl = a.exclude_dev != nullptr ? *a.exclude_dev : a.exclude;

  // Stage the thread's 32 values in registers (chunk = 8 x 256 float4 groups): value i of thread t
  // is column lo + ((i / 4) * kSelThreads + t) * 4 + i % 4, ascending in i.
  float vals[32];
#pragma unroll
  for (int k = 0; k < kSelChunk / (kSelThreads * 4); ++k) {
    const int base = lo + (k * kSelThreads + tid) * 4;
    if (vec && base + 4 <= hi) {
      const float4 q = __ldcs(reinterpret_cast<const float4*>(x + base));
      vals[k * 4 + 0] = q.x;
      vals[k * 4 + 1] = q.y;
      vals[k * 4 + 2] = q.z;
      vals[k * 4 + 3] = q.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) vals[k * 4 + e] = base + e < hi ? x[base + e] : -INFINITY;
    }
  }
  // The excluded column (scored as -inf): only the thread holding it rewrites its slot.
  if (excl >= lo && excl < hi && (((excl - lo) >> 2) & (kSelThreads - 1)) == tid) {
    const int slot = (((excl - lo) >> 2) / kSelThreads) * 4 + ((excl - lo) & 3);
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i == slot) vals[i] = -INFINITY;
  }
  // Chunk maximum (NaN ignored, as a > comparison ignores it), then its first column: only the
  // threads that hold the maximum look for it.
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; ++i) m = fmaxf(m, vals[i]);
  const float own_max = m;
  __shared__ float s_m[kSelThreads / 32];
  __shared__ int s_i[kSelThreads / 32];
  __shared__ double s_s[kSelThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) s_m[tid >> 5] = m;
  __syncthreads();
  float bm = s_m[0];
  for (int w = 1; w < kSelThreads / 32; ++w) bm = fmaxf(bm, s_m[w]);
  int idx = INT_MAX;
  if (bm != -INFINITY && own_max == bm) {
#pragma unroll
    for (int i = 31; i >= 0; --i)
      if (vals[i] == bm) idx = lo + ((i >> 2) * kSelThreads + tid) * 4 + (i & 3);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) idx = min(idx, __shfl_xor_sync(0xffffffffu, idx, o));
  if ((tid & 31) == 0) s_i[tid >> 5] = idx;
  __syncthreads();
  int bi = s_i[0];
  for (int w = 1; w < kSelThreads / 32; ++w) bi = min(bi, s_i[w]);

  const double samp_t = !kSample ? 0.0 : (a.sample_t_dev != nullptr ? *a.sample_t_dev : a.sample_t);
  const bool sample = kSample && (a.mode == SEL_SAMPLE || (a.mode == SEL_MAXPROB && a.sample_t_dev != nullptr)) && samp_t > 0.0;
  __shared__ double s_k1[kSelThreads / 32], s_k2[kSelThreads / 32];
  __shared__ int s_ki[kSelThreads / 32];
  double k1 = -INFINITY, k2 = -INFINITY;
  int ki = INT_MAX;
  if (sample) {
    const unsigned long long seed = a.sample_seed_dev != nullptr ? *a.sample_seed_dev : a.sample_seed;
    const int fwd = a.sample_forward_dev != nullptr ? *a.sample_forward_dev : a.sample_forward;
    const unsigned long long rk = sample_row_key(seed, fwd, a.positions[r]);
    // This thread's values in ascending index order: strict > keeps the lowest index among equals.
#pragma unroll
    for (int k = 0; k < kSelChunk / (kSelThreads * 4); ++k) {
      const int base = lo + (k * kSelThreads + tid) * 4;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (base + e >= hi) continue;
        const double key = __dadd_rn(static_cast<double>(vals[k * 4 + e]),
                                     __dmul_rn(samp_t, static_cast<double>(sample_gumbel(rk, base + e))));
        if (key > k1) { k2 = k1; k1 = key; ki = base + e; }
        else if (key > k2) { k2 = key; }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const double v1 = __shfl_xor_sync(0xffffffffu, k1, o);
      const int j1 = __shfl_xor_sync(0xffffffffu, ki, o);
      const double v2 = __shfl_xor_sync(0xffffffffu, k2, o);
      top2_merge(k1, ki, k2, v1, j1, v2);
    }
    if ((tid & 31) == 0) { s_k1[tid >> 5] = k1; s_ki[tid >> 5] = ki; s_k2[tid >> 5] = k2; }
    __syncthreads();
    k1 = s_k1[0]; ki = s_ki[0]; k2 = s_k2[0];
    for (int w = 1; w < kSelThreads / 32; ++w) top2_merge(k1, ki, k2, s_k1[w], s_ki[w], s_k2[w]);
  }

  const double inv_t = sample ? 1.0 : sel_inv_t(a.temperature);
  const double amax = sel_adjust(static_cast<double>(bm), inv_t);
  // sum of exp(adjusted - chunk max): a -inf (or NaN) term is clamped to exp(-708), about 3e-308,
  // which leaves a sum holding the chunk maximum's exp(0) = 1 unchanged; a chunk with no finite
  // value sums nothing.
  double sum = 0.0;
  double ent = 0.0;  // kEntropy: sum e z, z = max(a - chunk max, -708) (a clamped term adds about -2e-305)
  if (bm != -INFINITY) {
    if (!kEntropy && inv_t == 1.0) {  // no temperature (max-prob, sampled): a = x exactly
#pragma unroll
      for (int i = 0; i < 32; ++i) sum += exp_nonpos_clamped(static_cast<double>(vals[i]) - amax);
    } else if constexpr (kEntropy) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const double z = fmax(sel_adjust(static_cast<double>(vals[i]), inv_t) - amax, -708.0);
        const double e = exp_nonpos_core(z);  // exp_nonpos_clamped of the same argument
        sum += e;
        ent = fma(e, z, ent);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) sum += exp_nonpos_clamped(sel_adjust(static_cast<double>(vals[i]), inv_t) - amax);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((tid & 31) == 0) s_s[tid >> 5] = sum;
  __shared__ double s_e[kSelThreads / 32];
  if constexpr (kEntropy) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ent += __shfl_xor_sync(0xffffffffu, ent, o);
    if ((tid & 31) == 0) s_e[tid >> 5] = ent;
  }
  __syncthreads();
  __shared__ int s_last;
  if (tid == 0) {
    double bs = 0.0;
    for (int w = 0; w < kSelThreads / 32; ++w) bs += s_s[w];
    const int slot = r * a.nchunks + c;
    a.part_max[slot] = bm;
    a.part_idx[slot] = bi;
    a.part_sum[slot] = bs;
    if constexpr (kEntropy) {
      double be = 0.0;
      for (int w = 0; w < kSelThreads / 32; ++w) be += s_e[w];
      a.part_ent[slot] = be;
    }
    if (sample) {
      a.part_skey[slot] = k1;
      a.part_sidx[slot] = ki;
      a.part_skey2[slot] = k2;
    }
    __threadfence();
    const int old = atomicAdd(&a.counters[r], 1);
    s_last = (old == a.nchunks - 1);
  }
  __syncthreads();
  if (!s_last || tid != 0) return;
  __threadfence();
  // Merge the row's chunks in chunk order.
  float gm = -INFINITY;
  int gi = INT_MAX;
  for (int k = 0; k < a.nchunks; ++k) argmax_merge(gm, gi, __ldcg(&a.part_max[r * a.nchunks + k]), __ldcg(&a.part_idx[r * a.nchunks + k]));
  const double gam = sel_adjust(static_cast<double>(gm), inv_t);
  double S = 0.0;
  double row_ent = 0.0;  // kEntropy: sum e (a - m) over the row
  for (int k = 0; k < a.nchunks; ++k) {
    const float cm = __ldcg(&a.part_max[r * a.nchunks + k]);
    const double cs = __ldcg(&a.part_sum[r * a.nchunks + k]);
    if (cm == -INFINITY) continue;
    const double cam = sel_adjust(static_cast<double>(cm), inv_t);
    const double f = (cam == gam) ? 1.0 : exp_nonpos(cam - gam);
    S += (cam == gam) ? cs : cs * f;
    if constexpr (kEntropy) {
      // chunk terms e_c z_c with e = e_c f and a - m = z_c + (cam - gam): both parts <= 0
      const double ce = __ldcg(&a.part_ent[r * a.nchunks + k]);
      row_ent += (cam == gam) ? ce : f * fma(cam - gam, cs, ce);
    }
  }
  if (sample) {
    double g1 = -INFINITY, g2 = -INFINITY;
    int gj = INT_MAX;
    for (int k = 0; k < a.nchunks; ++k)
      top2_merge(g1, gj, g2, __ldcg(&a.part_skey[r * a.nchunks + k]), __ldcg(&a.part_sidx[r * a.nchunks + k]),
                 __ldcg(&a.part_skey2[r * a.nchunks + k]));
    if (gj < 0 || gj >= a.vocab) gj = gi;  // every key -inf (an all -inf row): keep the first max
    a.token[r] = gj;
    const float xt = (gj == excl) ? -INFINITY : x[gj];
    a.conf[r] = __ddiv_rn(exp_nonpos(static_cast<double>(xt) - gam), S);
    if (a.row_tie != nullptr) a.row_tie[r] = (g1 - g2 <= kSampleTieScale * samp_t) ? TIE_NEAR_BIT : 0;
    a.counters[r] = 0;
    return;
  }
  if (a.row_tie != nullptr) a.row_tie[r] = 0;
  a.token[r] = gi;
  if (a.mode == SEL_MAXPROB || a.mode == SEL_SAMPLE) {
    a.conf[r] = 1.0 / S;
  } else {
    a.row_amax[r] = static_cast<double>(gm);
    a.row_sum[r] = S;
    if constexpr (kEntropy) a.part_ent[r * a.nchunks] = row_ent / S - log(S);  // every chunk value is read
  }
  a.counters[r] = 0;
}

// Pass 2 (entropy): C / eps = sum p log1p(eps / p) / eps in float32 per logit, then the row's
// H = (exact part from pass 1) + eps (C / eps). With d = log2(p / eps) and q = 2^-|d| in (0, 1]:
//   d >= 0 (p >= eps): p log1p(eps / p) / eps = log1p(q) / q;
//   d <  0 (p <  eps): p log1p(eps / p) / eps = q (log1p(q) + |d| ln 2)   (log(eps / p) = |d| ln 2).
// d = (x - max x) (log2(e) / T) - log2(S) - log2(eps), the two constants split into float32 head
// and tail so that only the rounding of d itself (relative 6e-8, about 1e-6 on q) is left; |d| is
// capped at 200, and q below 2^-126 flushes to 0 (such a term is below 1e-36 and dropped). A -inf
// logit (the excluded column, p = 0 in the reference) and a NaN one land on that cap and add nothing.
// log1p(q) = 2 atanh(s) = 2 s P(s^2) with s = q / (2 + q) <= 1/3 and P the atanh series through
// s^14 / 15 (truncation below 2e-8 relative), so log1p(q) / q = 2 P / (2 + q): no division by q and
// no cancellation at small q. 2^w and 1 / (2 + q) are the hardware approximations (ex2.approx,
// rcp.approx: relative error within a few 2^-23).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__global__ void __launch_bounds__(kSelThreads) sel_entropy_kernel(const SelArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  int rows_valid = a.rows;
  if (a.rows_dev != nullptr) rows_valid = min(rows_valid, *a.rows_dev);
  const int r = blockIdx.y;
  if (r >= rows_valid) return;
  const int c = blockIdx.x;
  const int src = a.row_index != nullptr ? a.row_index[r] : r;
  const float* x = a.logits + static_cast<int64_t>(src) * a.ld;
  const int lo = c * a.chunk;
  const int hi = min(a.vocab, lo + a.chunk);
  const int tid = threadIdx.x;
  const float gm = static_cast<float>(a.row_amax[r]);
  const double S = a.row_sum[r];
  const int excl = a.exclude_dev != nullptr ? *a.exclude_dev : a.exclude;
  constexpr double kLog2e = 1.4426950408889634074;
  constexpr double kLog2Eps = -33.219280948873623479;  // log2(1e-10)
  constexpr float kLn2 = 0.693147180559945309f;
  const double s1 = sel_inv_t(a.temperature) * kLog2e;
  const float s1h = static_cast<float>(s1), s1l = static_cast<float>(s1 - static_cast<double>(s1h));
  const double c0 = -(log2(S) + kLog2Eps);
  const float c0h = static_cast<float>(c0), c0l = static_cast<float>(c0 - static_cast<double>(c0h));
  // The thread's columns as in sel_pass1_kernel (float4 groups lo + (k * kSelThreads + t) * 4).
  const bool vec = ((a.ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0);
  double acc = 0.0;
#pragma unroll 2
  for (int k = 0; k < kSelChunk / (kSelThreads * 4); ++k) {
    const int base = lo + (k * kSelThreads + tid) * 4;
    float v[4];
    if (vec && base + 4 <= hi) {
      const float4 q4 = __ldcs(reinterpret_cast<const float4*>(x + base));
      v[0] = q4.x;
      v[1] = q4.y;
      v[2] = q4.z;
      v[3] = q4.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = base + e < hi ? x[base + e] : -INFINITY;
    }
    float g = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float dx = (base + e == excl ? -INFINITY : v[e]) - gm;
      const float d = fmaf(dx, s1h, c0h) + fmaf(dx, s1l, c0l);
      const float w = fmaxf(-fabsf(d), -200.0f);
      const float q = ex2_approx(w);
      const float rq = rcp_approx(2.0f + q);
      const float sq = q * rq;
      const float t = sq * sq;
      float P = 1.0f / 15.0f;
      P = fmaf(P, t, 1.0f / 13.0f);
      P = fmaf(P, t, 1.0f / 11.0f);
      P = fmaf(P, t, 1.0f / 9.0f);
      P = fmaf(P, t, 1.0f / 7.0f);
      P = fmaf(P, t, 1.0f / 5.0f);
      P = fmaf(P, t, 1.0f / 3.0f);
      P = fmaf(P, t, 1.0f);
      g += d >= 0.0f ? 2.0f * rq * P : q * fmaf(2.0f * sq, P, -w * kLn2);
    }
    acc += static_cast<double>(g);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ double s_s[kSelThreads / 32];
  __shared__ int s_last;
  if ((tid & 31) == 0) s_s[tid >> 5] = acc;
  __syncthreads();
  if (tid == 0) {
    double bs = 0.0;
    for (int w = 0; w < kSelThreads / 32; ++w) bs += s_s[w];
    a.part_sum[r * a.nchunks + c] = bs;
    __threadfence();
    const int old = atomicAdd(&a.counters[r], 1);
    s_last = (old == a.nchunks - 1);
  }
  __syncthreads();
  if (!s_last || tid != 0) return;
  __threadfence();
  double Ce = 0.0;
  for (int k = 0; k < a.nchunks; ++k) Ce += __ldcg(&a.part_sum[r * a.nchunks + k]);
  const double H = __ldcg(&a.part_ent[r * a.nchunks]) + 1e-10 * Ce;
  a.conf[r] = static_cast<double>(static_cast<float>(H));
  a.counters[r] = 0;
}

// Batched choice over per-item confidence runs (the selector's output for each batch item's
// masked positions, row offsets[b] .. offsets[b + 1]). One warp per item.
//   top-k (_topk_count_choices, python/src/edllm/backends/diffusion_runtime.py:290-299): the k
//     highest confidences, the lowest row first among equal values;
//   threshold (_threshold_choices, :302-314): every row with conf >= tau, else the first argmax.
// chosen[row] = 1 for committed rows, 0 otherwise. tie[b] certifies the decision like the device
// decode policy: TIE bit 1 (near) when the k-th / (k+1)-th gap, or any |conf - tau| (and, without a
// hit, the top-1 / top-2 gap), is within tie_rel relative; bit 2 (exact) when those values are
// equal. Those are the only items where NumPy's unstable argsort or its own last-bit rounding of
// the confidence may decide differently.
enum ChoiceMode : int { CHOICE_TOPK = 0, CHOICE_THRESHOLD = 1 };

__device__ __forceinline__ void warp_best(double v, int i, double& bv, int& bi) {
  bv = v;
  bi = i;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double v2 = __shfl_xor_sync(0xffffffffu, bv, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v2 > bv || (v2 == bv && i2 < bi)) {
      bv = v2;
      bi = i2;
    }
  }
}

__global__ void __launch_bounds__(32) sel_choose_kernel(const double* __restrict__ conf, const int* __restrict__ offsets,
                                                        int mode, int k, double tau, double tie_rel, int* chosen, int* tie) {
  const int b = blockIdx.x;
  const int lane = threadIdx.x;
  const int r0 = offsets[b], r1 = offsets[b + 1];
  const int n = r1 - r0;
  for (int i = lane; i < n; i += 32) chosen[r0 + i] = 0;
  __syncwarp();
  int flag = 0;
  if (n <= 0) {
    if (lane == 0) tie[b] = 0;
    return;
  }
  if (mode == CHOICE_TOPK) {
    const int kk = min(k, n);
    double prev = 0.0;
    for (int round = 0; round <= kk && round < n; ++round) {
      // best remaining row: lane-local scan, then warp reduction (lowest index among equals)
      double bv = -INFINITY;
      int bi = INT_MAX;
      for (int i = lane; i < n; i += 32) {
        if (chosen[r0 + i]) continue;
        const double v = conf[r0 + i];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
      }
      double wv;
      int wi;
      warp_best(bv, bi, wv, wi);
      if (round < kk) {
        if (lane == 0) chosen[r0 + wi] = 1;
        __syncwarp();
        prev = wv;
      } else {
        // rank k + 1: certify the cut
        if (wv == prev) flag |= 2;
        else if (!(prev - wv > tie_rel * fabs(prev))) flag |= 1;
      }
    }
  } else {
    int hits = 0;
    for (int i = lane; i < n; i += 32) {
      const double v = conf[r0 + i];
      if (v >= tau) {
        chosen[r0 + i] = 1;
        ++hits;
      }
      if (!(fabs(v - tau) > tie_rel * fabs(tau))) flag |= (v == tau) ? 2 : 1;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      hits += __shfl_xor_sync(0xffffffffu, hits, o);
      flag |= __shfl_xor_sync(0xffffffffu, flag, o);
    }
    if (hits == 0) {
      double bv = -INFINITY, sv = -INFINITY;
      int bi = INT_MAX;
      for (int i = lane; i < n; i += 32) {
        const double v = conf[r0 + i];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
      }
      double wv;
      int wi;
      warp_best(bv, bi, wv, wi);
      // second best (excluding the winner's row)
      for (int i = lane; i < n; i += 32)
        if (i != wi) sv = fmax(sv, conf[r0 + i]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sv = fmax(sv, __shfl_xor_sync(0xffffffffu, sv, o));
      if (lane == 0) chosen[r0 + wi] = 1;
      if (n > 1) {
        if (sv == wv) flag |= 2;
        else if (!(wv - sv > tie_rel * fabs(wv))) flag |= 1;
      }
    }
  }
  if (lane == 0) tie[b] = flag;
}

// Negative-entropy confidence with a top-p nucleus (_entropy_confidence with top_p,
// python/src/edllm/backends/diffusion_runtime.py:90-114, _top_p_filter :358-370, _softmax :373-378),
// one CTA per row:
//   a = f64(x) / T (T > 0); the excluded token (MASK) is -inf;
//   sort a descending, cum = cumsum(softmax(sorted)); drop every entry with cum > top_p except the
//   first; p' = softmax over the kept entries; conf = f32(sum p' log(p' + 1e-10)); token = argmax p'.
// The kept set is found without sorting. v_b, the first dropped value, is the largest logit whose
// inclusive mass (the p of every entry >= v_b) exceeds top_p. Every entry above v_b is kept, and of
// the m copies of v_b the first c are, c = #{i in 1..m : above + i * p(v_b) <= top_p} (at least one
// when v_b is the maximum). Which copies the reference's unstable sort puts first does not change
// the entropy, since the copies are equal, nor the token unless v_b is a tied maximum.
//
// Passes over the row (one CTA per row, about one CTA per SM so the rows in flight stay in L2):
//   1. max logit and its first index;
//   2. S = sum exp(a - max) (f64, per-thread then block order) and a histogram of that mass over
//      the distance from the maximum, max - a, in 1/8 steps (f32, per-warp: the bins spread the
//      vocabulary, so updates rarely collide; the histogram only places the list cut, below);
//   3. the keys of every entry up to one bin past the bin where the cumulative mass crosses
//      top_p * S, in index order, into a shared-memory list. Every kept entry and every copy of
//      v_b is on it, and every entry off it lies below v_b.
// v_b is then located exactly by a radix search over the order-preserving 32-bit keys of the list
// (four 8-bit levels, each accumulating the mass of the keys under the current prefix per digit and
// descending into the digit where the cumulative mass from the top crosses top_p * S), and the
// nucleus normaliser and entropy are summed over the list. When the list would overflow (a flat
// distribution whose nucleus holds most of the vocabulary), or its f64 mass does not reach
// top_p * S (the f32 histogram misplaced the cut), the same radix search and sums run over the whole
// row instead.
// tie[r]: bit 2 when the kept copies are a strict subset of a tied maximum (the reference's sort
// order picks the token); bit 1 when a cumulative mass at the cut is within tie_rel of top_p (the
// reference's own summation order may decide the other way there).
struct ToppArgs {
  const float* logits;
  int64_t ld;
  const int* row_index;  // optional gather
  int rows;
  const int* rows_dev;   // optional device-side row count
  int vocab;
  double temperature;    // <= 0: no scaling
  double top_p;          // >= 1: no nucleus
  int exclude;           // -1 for none
  double tie_rel;
  double* conf;
  int* token;
  int* tie;              // optional
};

constexpr int kToppThreads = 512;
constexpr int kToppWarps = kToppThreads / 32;
constexpr int kToppBins = 256;           // distance-from-max bins of 1/8 (the last one open-ended)
constexpr double kToppBinScale = 8.0;
constexpr int kToppList = 24576;         // candidate keys held in shared memory
constexpr size_t kToppSmemBytes = static_cast<size_t>(kToppList) * 4 + static_cast<size_t>(kToppWarps) * kToppBins * 4;

__device__ __forceinline__ uint32_t f32_order_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float f32_from_order_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

template <typename T>
__device__ __forceinline__ T topp_block_sum(T v, T* red, int lane, int warp) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  T t = T(0);
  for (int w = 0; w < kToppWarps; ++w) t += red[w];
  __syncthreads();
  return t;
}

// Distance bin of logit v below the maximum gm, in f32 (only consistency between the passes and
// monotonicity matter: the exact cut is found afterwards from the keys).
__device__ __forceinline__ int topp_bin(float gm, float v, float scale) {
  const float d = (gm - v) * scale;
  return d < static_cast<float>(kToppBins - 1) ? static_cast<int>(d) : kToppBins - 1;
}

// Shared state of one row's search.
struct ToppShared {
  double hist[256];
  int hcnt[256];
  double red_d[kToppWarps];
  float red_f[kToppWarps];
  int red_i[kToppWarps];
  int warp_tot[kToppWarps + 1];
  uint32_t prefix, mask;
  double above;
  int count, c, flag, n_list;
};

// Radix search for v_b over the keys key_at(i), i < n (valid(i) false skips an entry); returns
// (in sh) prefix = key of v_b, above = mass strictly above it, count = its multiplicity.
template <typename KeyAt, typename Valid>
__device__ void topp_radix(ToppShared& sh, int n, KeyAt key_at, Valid valid, double invT, double am, double limit) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, pmask = 0;
  double above = 0.0;
  for (int level = 0; level < 4; ++level) {
    const int shift = 24 - 8 * level;
    for (int i = tid; i < 256; i += kToppThreads) { sh.hist[i] = 0.0; sh.hcnt[i] = 0; }
    __syncthreads();
    for (int i = tid; i < n; i += kToppThreads) {
      if (!valid(i)) continue;
      const uint32_t k = key_at(i);
      if ((k & pmask) != prefix) continue;
      const double e = exp_nonpos(static_cast<double>(f32_from_order_key(k)) * invT - am);
      const int d = static_cast<int>((k >> shift) & 255u);
      atomicAdd(&sh.hist[d], e);
      if (level == 3) atomicAdd(&sh.hcnt[d], 1);
    }
    __syncthreads();
    if (tid == 0) {
      double cum = above;
      int d = 255;
      for (; d > 0; --d) {
        if (cum + sh.hist[d] > limit) break;
        cum += sh.hist[d];
      }
      sh.above = cum;
      sh.count = sh.hcnt[d];
      sh.prefix = prefix | (static_cast<uint32_t>(d) << shift);
      sh.mask = pmask | (0xFFu << shift);
    }
    __syncthreads();
    prefix = sh.prefix;
    pmask = sh.mask;
    above = sh.above;
    __syncthreads();
  }
}

// f(i, x[i]) for every i < V; each thread keeps 16 loads in flight (the row is read from L2 or
// HBM, so one outstanding load per thread would leave the pass latency-bound). A thread visits
// its indices in increasing order.
template <typename F>
__device__ __forceinline__ void topp_row_foreach(const float* __restrict__ x, int V, F f) {
  const int tid = threadIdx.x;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (V & 3) == 0) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int V4 = V >> 2;
    constexpr int U = 4;
    int j = tid;
    for (; j + (U - 1) * kToppThreads < V4; j += U * kToppThreads) {
      float4 t[U];
#pragma unroll
      for (int u = 0; u < U; ++u) t[u] = __ldg(x4 + j + u * kToppThreads);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = 4 * (j + u * kToppThreads);
        f(i, t[u].x);
        f(i + 1, t[u].y);
        f(i + 2, t[u].z);
        f(i + 3, t[u].w);
      }
    }
    for (; j < V4; j += kToppThreads) {
      const float4 t = __ldg(x4 + j);
      f(4 * j, t.x);
      f(4 * j + 1, t.y);
      f(4 * j + 2, t.z);
      f(4 * j + 3, t.w);
    }
  } else {
    constexpr int U = 8;
    int i = tid;
    for (; i + (U - 1) * kToppThreads < V; i += U * kToppThreads) {
      float t[U];
#pragma unroll
      for (int u = 0; u < U; ++u) t[u] = __ldg(x + i + u * kToppThreads);
#pragma unroll
      for (int u = 0; u < U; ++u) f(i + u * kToppThreads, t[u]);
    }
    for (; i < V; i += kToppThreads) f(i, __ldg(x + i));
  }
}

__global__ void __launch_bounds__(kToppThreads) sel_topp_entropy_kernel(const ToppArgs a) {
  extern __shared__ __align__(16) uint8_t topp_smem[];
  uint32_t* list = reinterpret_cast<uint32_t*>(topp_smem);
  float* whist = reinterpret_cast<float*>(topp_smem + static_cast<size_t>(kToppList) * 4);
  __shared__ ToppShared sh;
  griddep_wait();
  griddep_launch_dependents();
  const int r = blockIdx.x;
  const int rows = a.rows_dev != nullptr ? min(a.rows, *a.rows_dev) : a.rows;
  if (r >= rows) return;
  const int src = a.row_index != nullptr ? a.row_index[r] : r;
  const float* x = a.logits + static_cast<int64_t>(src) * a.ld;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // x / T taken as x * (1 / T): the two differ in the last f64 bit at most, far below the f32 result
  const double invT = a.temperature > 0.0 ? 1.0 / a.temperature : 1.0;
  const bool nucleus = a.top_p < 1.0;
  const int V = a.vocab, ex = a.exclude;

  // 1. max logit and its first index
  float m = -INFINITY;
  int mi = INT_MAX;
  topp_row_foreach(x, V, [&](int i, float v) {
    if (i != ex && v > m) { m = v; mi = i; }
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, mi, o);
    argmax_merge(m, mi, m2, i2);
  }
  if (lane == 0) { sh.red_f[warp] = m; sh.red_i[warp] = mi; }
  for (int i = tid; i < kToppWarps * kToppBins; i += kToppThreads) whist[i] = 0.0f;
  __syncthreads();
  float gm = sh.red_f[0];
  int gmi = sh.red_i[0];
  for (int w = 1; w < kToppWarps; ++w) argmax_merge(gm, gmi, sh.red_f[w], sh.red_i[w]);
  const double am = static_cast<double>(gm) * invT;
  const float bin_scale = static_cast<float>(kToppBinScale * invT);
  __syncthreads();

  // 2. S and the distance histogram
  double part = 0.0;
  float* my_hist = whist + warp * kToppBins;
  topp_row_foreach(x, V, [&](int i, float v) {
    if (i == ex) return;
    const double e = exp_nonpos(static_cast<double>(v) * invT - am);
    part += e;
    if (nucleus) {
      const int bin = topp_bin(gm, v, bin_scale);
      if (bin < kToppBins - 1) atomicAdd(&my_hist[bin], static_cast<float>(e));  // the open last bin is never read
    }
  });
  const double S = topp_block_sum(part, sh.red_d, lane, warp);
  const double limit = a.top_p * S;

  // 3. candidate list: every entry up to one bin past the crossing bin, in index order
  bool use_list = false;
  if (nucleus) {
    if (tid == 0) {
      double cum = 0.0;
      int b = 0;
      for (; b < kToppBins - 1; ++b) {
        double hb = 0.0;
        for (int w = 0; w < kToppWarps; ++w) hb += static_cast<double>(whist[w * kToppBins + b]);
        cum += hb;
        if (cum > limit) break;
      }
      sh.c = min(b + 1, kToppBins - 1);  // last bin on the list
      sh.n_list = 0;
    }
    __syncthreads();
    const int last_bin = sh.c;
    int n = 0;
    bool overflow = false;
    if (last_bin < kToppBins - 1) {
      // thread t owns 8 consecutive entries of each 4096-entry chunk; a block scan of the per-thread
      // counts writes the chunk's keys in index order
      constexpr int G = 8;
      for (int base = 0; base < V && !overflow; base += G * kToppThreads) {
        const int i0 = base + G * tid;
        float v[G];
        if (i0 + G <= V && (reinterpret_cast<uintptr_t>(x + i0) & 15) == 0) {
          const float4 t0 = __ldg(reinterpret_cast<const float4*>(x + i0));
          const float4 t1 = __ldg(reinterpret_cast<const float4*>(x + i0) + 1);
          v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w;
          v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
        } else {
#pragma unroll
          for (int g = 0; g < G; ++g) v[g] = i0 + g < V ? __ldg(x + i0 + g) : -INFINITY;
        }
        unsigned takes = 0;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const int i = i0 + g;
          if (i < V && i != ex && topp_bin(gm, v[g], bin_scale) <= last_bin) takes |= 1u << g;
        }
        const int cnt = __popc(takes);
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        if (lane == 31) sh.warp_tot[warp] = incl;
        __syncthreads();
        if (tid == 0) {
          int acc = 0;
          for (int w = 0; w < kToppWarps; ++w) {
            const int t = sh.warp_tot[w];
            sh.warp_tot[w] = acc;
            acc += t;
          }
          sh.warp_tot[kToppWarps] = acc;
        }
        __syncthreads();
        const int tot = sh.warp_tot[kToppWarps];
        if (n + tot > kToppList) {
          overflow = true;
        } else {
          int pos = n + sh.warp_tot[warp] + incl - cnt;
#pragma unroll
          for (int g = 0; g < G; ++g)
            if (takes & (1u << g)) list[pos++] = f32_order_key(v[g]);
        }
        n += tot;
        __syncthreads();
      }
    } else {
      overflow = true;
    }
    use_list = !overflow;
    if (use_list) {
      // the list must hold the crossing: its own mass has to exceed the limit
      double lm = 0.0;
      for (int i = tid; i < n; i += kToppThreads) lm += exp_nonpos(static_cast<double>(f32_from_order_key(list[i])) * invT - am);
      use_list = topp_block_sum(lm, sh.red_d, lane, warp) > limit;
    }
    if (use_list) {
      topp_radix(sh, n, [&](int i) { return list[i]; }, [](int) { return true; }, invT, am, limit);
      if (tid == 0) sh.n_list = n;
    } else {
      topp_radix(sh, V, [&](int i) { return f32_order_key(x[i]); }, [&](int i) { return i != ex; }, invT, am, limit);
    }
  }
  const uint32_t vb = nucleus ? sh.prefix : 0u;
  // kept copies of v_b and the certification flags
  if (tid == 0) {
    int c = 0, flag = 0;
    if (nucleus) {
      const double above = sh.above;
      const int count = sh.count;
      const double e = exp_nonpos(static_cast<double>(f32_from_order_key(vb)) * invT - am);
      while (c < count && above + static_cast<double>(c + 1) * e <= limit) ++c;
      if (above == 0.0 && c == 0) c = 1;
      const double tol = a.tie_rel * limit;
      if (!(fabs(above + static_cast<double>(c) * e - limit) > tol)) flag |= 1;
      if (c < count && !(fabs(above + static_cast<double>(c + 1) * e - limit) > tol)) flag |= 1;
      if (above == 0.0 && c < count) flag |= 2;
    }
    sh.c = c;
    sh.flag = flag;
  }
  __syncthreads();
  const int c = sh.c;
  const double e_vb = nucleus ? exp_nonpos(static_cast<double>(f32_from_order_key(vb)) * invT - am) : 0.0;

  // normaliser and entropy over the kept entries (the list, or the whole row)
  const int n_src = use_list ? sh.n_list : V;
  auto kept_value = [&](int i, float* v) -> bool {
    if (use_list) {
      const uint32_t k = list[i];
      *v = f32_from_order_key(k);
      return k > vb;
    }
    if (i == ex) return false;
    *v = x[i];
    return !nucleus || f32_order_key(*v) > vb;
  };
  double sk = 0.0;
  for (int i = tid; i < n_src; i += kToppThreads) {
    float v;
    if (kept_value(i, &v)) sk += exp_nonpos(static_cast<double>(v) * invT - am);
  }
  double Sk = topp_block_sum(sk, sh.red_d, lane, warp);
  Sk += static_cast<double>(c) * e_vb;
  double h = 0.0;
  for (int i = tid; i < n_src; i += kToppThreads) {
    float v;
    if (kept_value(i, &v)) {
      const double pv = exp_nonpos(static_cast<double>(v) * invT - am) / Sk;
      h += pv * log(pv + 1e-10);
    }
  }
  double H = topp_block_sum(h, sh.red_d, lane, warp);
  if (tid == 0) {
    if (c > 0) {
      const double pv = e_vb / Sk;
      H += static_cast<double>(c) * (pv * log(pv + 1e-10));
    }
    a.conf[r] = static_cast<double>(static_cast<float>(H));
    a.token[r] = gmi;
    if (a.tie != nullptr) a.tie[r] = sh.flag;
  }
}

}  // namespace drt
