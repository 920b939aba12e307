// Full-canvas masked diffusion (Dream) with the entropy_count schedule, device side.
//
// One denoising step of EntropyCountStrategy (python/src/edllm/backends/diffusion_runtime.py:2079-2110)
// through run_decode_loop (:1829-1991):
//   plan:    frontier = every masked position >= prompt_len, ascending (MaskState.masked_positions,
//            :451-470); the transfer count k of this step (EntropyCountCommit.plan, :921-937) is
//            precomputed by the host: the masked count falls by exactly k per proceeding step, so
//            the whole schedule follows from the initial count.
//   forward: the whole canvas, bidirectional attention; logits of position p are the raw row
//            max(p - 1, 0) (dream_ar_shift, mlx_ops.shift_logits_for_dream :157-159).
//   score:   NegEntropy with temperature and top_p, MASK excluded (sel_topp_entropy_kernel).
//   select:  the top-k rows by confidence (_topk_count_choices, :290-299: argsort(-conf)[:k]).
//   commit:  canvas[frontier[i]] = token[i] for the chosen rows.
// The device picks equal confidences in ascending row order; the reference's argsort is not
// stable, so a cut through equal confidences is flagged (DRT_TIE_EXACT) rather than matched.
#pragma once
#include "common.cuh"
#include "policy.cuh"

namespace drt {

constexpr int kDreamThreads = 1024;
constexpr int kDreamMaxFrontier = 4096;  // rank staging in shared memory

struct DreamState {
  int canvas_len, prompt_len, mask_id;
  int n_proceed;        // proceeding steps in the schedule
  int iter;             // proceeding steps done
  int n_frontier;       // masked positions of this step
  int k;                // transfer count of this step
  int forward_count, committed_count, near_tie_steps, exact_tie_steps;
  int trace_cap;
  int shift;            // dream_ar_shift: position p is scored from row max(p - 1, 0), else row p
};

// Block-wide exclusive prefix of a 0/1 flag per thread; returns the block total.
__device__ __forceinline__ int dream_block_scan(int flag, int* warp_tot, int* excl) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned bal = __ballot_sync(0xffffffffu, flag);
  if (lane == 0) warp_tot[warp] = __popc(bal);
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int w = 0; w < kDreamThreads / 32; ++w) {
      const int t = warp_tot[w];
      warp_tot[w] = acc;
      acc += t;
    }
    warp_tot[kDreamThreads / 32] = acc;
  }
  __syncthreads();
  *excl = warp_tot[warp] + __popc(bal & ((1u << lane) - 1u));
  const int total = warp_tot[kDreamThreads / 32];
  __syncthreads();
  return total;
}

// Frontier of this step: masked positions in [prompt_len, canvas_len), ascending, and the raw
// logits row each one reads.
__global__ void __launch_bounds__(kDreamThreads) dream_plan_kernel(DreamState* st, const int* __restrict__ canvas,
                                                                   int* __restrict__ frontier_pos,
                                                                   int* __restrict__ frontier_row,
                                                                   const int* __restrict__ k_list) {
  griddep_wait();
  __shared__ int warp_tot[kDreamThreads / 32 + 1];
  const int lo = st->prompt_len, hi = st->canvas_len, mask = st->mask_id;
  int n = 0;
  for (int base = lo; base < hi; base += kDreamThreads) {
    const int p = base + threadIdx.x;
    const int f = (p < hi && canvas[p] == mask) ? 1 : 0;
    int slot;
    const int tot = dream_block_scan(f, warp_tot, &slot);
    if (f && n + slot < kDreamMaxFrontier) {
      frontier_pos[n + slot] = p;
      frontier_row[n + slot] = st->shift ? (p > 0 ? p - 1 : 0) : p;
    }
    n += tot;
  }
  if (threadIdx.x == 0) {
    st->n_frontier = min(n, kDreamMaxFrontier);
    st->k = st->iter < st->n_proceed ? k_list[st->iter] : 0;
  }
  griddep_launch_dependents();
}

// Top-k by rank (conf descending, row ascending among equals), certification, commit, counters
// and the step trace.
__global__ void __launch_bounds__(kDreamThreads) dream_commit_kernel(DreamState* st, int* __restrict__ canvas,
                                                                     const int* __restrict__ frontier_pos,
                                                                     const double* __restrict__ conf,
                                                                     const int* __restrict__ token,
                                                                     const int* __restrict__ row_tie, double tie_rel,
                                                                     const int* __restrict__ step_of, StepTrace* trace) {
  griddep_wait();
  __shared__ double sc[kDreamMaxFrontier];
  __shared__ double cut[2];
  __shared__ int s_flag;
  const int n = st->n_frontier;
  const int k = min(st->k, n);
  if (threadIdx.x == 0) {
    s_flag = 0;
    cut[0] = cut[1] = 0.0;
  }
  for (int i = threadIdx.x; i < n; i += kDreamThreads) sc[i] = conf[i];
  __syncthreads();
  int flag = 0;
  for (int i = threadIdx.x; i < n; i += kDreamThreads) {
    const double v = sc[i];
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const double w = sc[j];
      rank += (w > v || (w == v && j < i)) ? 1 : 0;
    }
    const bool chosen = rank < k;
    if (rank == k - 1) cut[0] = v;
    if (rank == k) cut[1] = v;
    const int rt = row_tie != nullptr ? row_tie[i] : 0;
    flag |= rt & TIE_NEAR;                 // the row's confidence itself is uncertain
    if (chosen) {
      flag |= rt & TIE_EXACT;              // the committed token depends on the sort order
      canvas[frontier_pos[i]] = token[i];
    }
  }
  flag = __reduce_or_sync(0xffffffffu, flag);
  if ((threadIdx.x & 31) == 0 && flag) atomicOr(&s_flag, flag);
  __syncthreads();
  if (threadIdx.x == 0) {
    int f = s_flag;
    if (k > 0 && k < n) {
      const double a = cut[0], b = cut[1];
      if (a == b) f |= TIE_EXACT;
      else if (!(a - b > tie_rel * fabs(a))) f |= TIE_NEAR;
    }
    const int it = st->iter;
    if (trace != nullptr && it < st->trace_cap) {
      StepTrace* t = trace + it;
      t->step = step_of[it];
      t->n_frontier = n;
      t->n_chosen = k;
      t->tie = f;
      unsigned long long bits = 0ull;
      for (int i = 0; i < min(n, kMaxFrontier); ++i) {
        t->frontier_pos[i] = frontier_pos[i];
        t->token[i] = token[i];
        t->conf[i] = sc[i];
        int rank = 0;
        for (int j = 0; j < n; ++j) rank += (sc[j] > sc[i] || (sc[j] == sc[i] && j < i)) ? 1 : 0;
        if (rank < k) bits |= 1ull << i;
      }
      t->chosen_mask = bits;
    }
    st->forward_count += 1;
    st->committed_count += k;
    if (f & TIE_NEAR) st->near_tie_steps += 1;
    if (f & TIE_EXACT) st->exact_tie_steps += 1;
    st->iter = it + 1;
  }
  griddep_launch_dependents();
}

}  // namespace drt
