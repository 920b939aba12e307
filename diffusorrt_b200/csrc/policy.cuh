// Device-resident decode policy: the plan -> (forward, score) -> select -> commit loop of the
// reference run_decode_loop (python/src/edllm/backends/diffusion_runtime.py:1829-1991), kept
// on the GPU so a CUDA graph replays a whole denoising step with no host round trip.
//
// Plans (one warp):
//   BD3 fixed quota  (BD3FixedQuotaCommit.plan, diffusion_runtime.py:1270-1334): absolute
//     blocks (origin 0); steps_per_block rounds per block; quota divmod(initial masks, rounds);
//     EOS stops only at a block boundary; zero-quota rounds are SKIPs; window_end = block end.
//   Block threshold  (BlockThresholdCommit + _block_frontier_plan, :1023-1095): the first
//     block of the generated span that still has masks. rounds_cap > 0 adds a per-block round
//     budget (after that many rounds the block is left with its residual masks), which the
//     long-prefix benchmark configuration uses; rounds_cap = 0 is the reference rule.
//   D2F block pipeline (D2FBlockPipelineCommit.plan, :1609-1671; threshold rule, no revision
//     window): a window of prompt-relative blocks decoded together. Fully decoded blocks leave it
//     oldest-first (frozen); a committed EOS in the appended region stops appending; at most one
//     block joins per step, when the last appended block's decoded ratio is >= tau_add (the prompt
//     counts as 1.0); block j is fully activated when block j - 1's ratio is >= tau_act (ratios
//     never fall, so the reference's sticky flag is this test on the current canvas). The frontier
//     is every masked position of the unfrozen appended blocks; the window ends at the last one.
// Select (one warp) on the device scores (selector.cuh):
//   top-k   (_topk_count_choices, :290-299): the k highest confidences, lowest index first
//           among equals;
//   threshold (_threshold_choices, :302-314): conf >= tau, else the first argmax;
//   pipeline  (D2FBlockPipelineCommit.select, :1673-1704): per unfrozen appended block, the rows
//           with conf strictly > tau, else (fully activated blocks only) the block's first argmax.
// Each decision is certified: a ranking gap or threshold distance within tie_rel (relative)
// sets TIE_NEAR for the step, equal confidences across the decision set TIE_EXACT. Those are
// the only steps where the f64 device score may order rows differently from NumPy's.
#pragma once
#include "common.cuh"

namespace drt {

constexpr int kMaxFrontier = 64;
constexpr int kMaxFwdRows = 64;

enum PolicyKind : int { POL_BD3_FIXED_QUOTA = 0, POL_BLOCK_THRESHOLD = 1, POL_D2F_PIPELINE = 2 };
enum PlanAction : int { PLAN_PROCEED = 0, PLAN_SKIP = 1, PLAN_STOP = 2 };
enum TieFlag : int { TIE_NEAR = 1, TIE_EXACT = 2 };

struct DecodeState {
  // request constants
  int canvas_len, prompt_len, gen_len, block_size, mask_id, eos_id;
  int policy, steps_per_block, iteration_limit, rounds_cap;
  int exclude_token;  // scored as -inf by the selector (block threshold excludes MASK), -1 none
  double threshold;
  double tie_rel;
  double sample_t;                 // fixed quota: Gumbel temperature (0 = argmax), selector.cuh
  unsigned long long sample_seed;  // keys the draws with forward_count and the row's position
  int shift;                       // dream_ar_shift: position p is scored from forwarded row p - 1
  double add_threshold, activate_threshold;  // D2F pipeline: tau_add, tau_act
  // loop state
  int step, stopped, action, error;
  int cache_end;
  int fwd_pos0, fwd_rows, kv_len;
  int n_frontier;
  int frontier_pos[kMaxFrontier];
  int frontier_row[kMaxFrontier];
  int active_block, base, remainder, round;
  int block_index, rounds_on_block;
  int forward_count, committed_count, iteration_count;
  int near_tie_steps, exact_tie_steps, last_tie;
  // D2F pipeline: blocks [0, pipe_frozen) frozen, [pipe_frozen, pipe_appended) in the window;
  // bit j of pipe_act: block pipe_frozen + j fully activated this step
  int pipe_blocks, pipe_frozen, pipe_appended, pipe_eos;
  unsigned long long pipe_act;
  int trace_cap;
};

struct StepTrace {
  int step, n_frontier, n_chosen, tie;
  int frontier_pos[kMaxFrontier];
  int token[kMaxFrontier];
  double conf[kMaxFrontier];
  unsigned long long chosen_mask;
};

__device__ __forceinline__ void plan_none(DecodeState* st, int action) {
  st->action = action;
  st->fwd_rows = 0;
  st->n_frontier = 0;
  if (action == PLAN_STOP) st->stopped = 1;
}

// Masked positions of [lo, hi) in ascending order -> st->frontier_pos; returns the count.
__device__ __forceinline__ int collect_masked(DecodeState* st, const int* x, int lo, int hi) {
  const int lane = threadIdx.x & 31;
  int n = 0;
  for (int base = lo; base < hi; base += 32) {
    const int p = base + lane;
    const bool m = p < hi && x[p] == st->mask_id;
    const unsigned bal = __ballot_sync(0xffffffffu, m);
    if (m) {
      const int slot = n + __popc(bal & ((1u << lane) - 1u));
      if (slot < kMaxFrontier) st->frontier_pos[slot] = p;
    }
    n += __popc(bal);
  }
  return n;
}

// Masked positions of [lo, hi) appended to st->frontier_pos from slot n0; returns the count added.
__device__ __forceinline__ int collect_masked_from(DecodeState* st, const int* x, int lo, int hi, int n0) {
  const int lane = threadIdx.x & 31;
  int n = 0;
  for (int base = lo; base < hi; base += 32) {
    const int p = base + lane;
    const bool m = p < hi && x[p] == st->mask_id;
    const unsigned bal = __ballot_sync(0xffffffffu, m);
    if (m) {
      const int slot = n0 + n + __popc(bal & ((1u << lane) - 1u));
      if (slot < kMaxFrontier) st->frontier_pos[slot] = p;
    }
    n += __popc(bal);
  }
  return n;
}

__device__ __forceinline__ int count_equal(const int* x, int lo, int hi, int value) {
  const int lane = threadIdx.x & 31;
  int n = 0;
  for (int p = lo + lane; p < hi; p += 32) n += x[p] == value ? 1 : 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
  return n;
}

// D2F pipeline block j of the generated span: [lo, hi).
__device__ __forceinline__ void pipe_span(const DecodeState* st, int j, int* lo, int* hi) {
  *lo = st->prompt_len + j * st->block_size;
  *hi = min(*lo + st->block_size, st->canvas_len);
}

// Decoded ratio of pipeline block j, as the reference computes it: (total - masked) / total.
__device__ __forceinline__ double pipe_ratio(const DecodeState* st, const int* x, int j) {
  int lo, hi;
  pipe_span(st, j, &lo, &hi);
  const int masked = count_equal(x, lo, hi, st->mask_id);
  return static_cast<double>(hi - lo - masked) / static_cast<double>(hi - lo);
}

__device__ __forceinline__ bool any_equal(const int* x, int lo, int hi, int value) {
  const int lane = threadIdx.x & 31;
  bool hit = false;
  for (int p = lo + lane; p < hi; p += 32) hit |= (x[p] == value);
  return __any_sync(0xffffffffu, hit);
}

// One warp. Decides this step's frontier and forward rows.
__global__ void plan_kernel(DecodeState* st, const int* x) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x;
  __syncwarp();
  if (st->stopped || st->error) {
    if (lane == 0) plan_none(st, PLAN_STOP);
    return;
  }
  const int step = st->step;
  if (step >= st->iteration_limit) {
    if (lane == 0) plan_none(st, PLAN_STOP);
    return;
  }
  int frozen = 0, window_end = 0, nf = 0;
  if (st->policy == POL_BD3_FIXED_QUOTA) {
    const int spb = st->steps_per_block;
    if (step % spb == 0 && any_equal(x, st->prompt_len, st->canvas_len, st->eos_id)) {
      if (lane == 0) plan_none(st, PLAN_STOP);
      return;
    }
    if (!any_equal(x, st->prompt_len, st->canvas_len, st->mask_id)) {
      if (lane == 0) plan_none(st, PLAN_STOP);
      return;
    }
    const int bs = st->block_size;
    const int block_id = step / spb;
    const int first = st->prompt_len / bs;
    const int grid_start = (first + block_id) * bs;
    const int b_lo = max(st->prompt_len, grid_start);
    const int b_hi = min(st->canvas_len, grid_start + bs);
    nf = collect_masked(st, x, b_lo, b_hi);
    __syncwarp();
    if (lane == 0) {
      if (st->active_block != block_id) {
        st->active_block = block_id;
        st->base = nf / spb;
        st->remainder = nf % spb;
      }
      st->round = step % spb;
    }
    __syncwarp();
    const int quota = st->base + (st->round < st->remainder ? 1 : 0);
    if (nf == 0 || quota == 0) {
      if (lane == 0) plan_none(st, PLAN_SKIP);
      return;
    }
    frozen = b_lo;
    window_end = b_hi;
  } else if (st->policy == POL_D2F_PIPELINE) {
    int fz = st->pipe_frozen, ap = st->pipe_appended, eos = st->pipe_eos;
    // 1. freeze: fully decoded blocks leave the window, oldest first
    while (fz < ap) {
      int lo, hi;
      pipe_span(st, fz, &lo, &hi);
      if (count_equal(x, lo, hi, st->mask_id) > 0) break;
      ++fz;
    }
    // 2. a committed EOS anywhere in the appended region stops appending
    if (!eos && ap > 0) {
      int lo, hi;
      pipe_span(st, ap - 1, &lo, &hi);
      eos = any_equal(x, st->prompt_len, hi, st->eos_id) ? 1 : 0;
    }
    // 3. at most one new block, when the last appended block is decoded far enough
    if (ap < st->pipe_blocks && !eos) {
      const double last = ap == 0 ? 1.0 : pipe_ratio(st, x, ap - 1);
      if (last >= st->add_threshold) ++ap;
    }
    // 4. activation and the frontier over the unfrozen appended blocks
    unsigned long long act = 0ull;
    bool over = ap - fz > 64;
    for (int j = fz; j < ap && !over; ++j) {
      const double prev = j == 0 ? 1.0 : pipe_ratio(st, x, j - 1);
      if (prev >= st->activate_threshold) act |= 1ull << (j - fz);
      int lo, hi;
      pipe_span(st, j, &lo, &hi);
      nf += collect_masked_from(st, x, lo, hi, nf);
    }
    __syncwarp();
    if (lane == 0) {
      st->pipe_frozen = fz;
      st->pipe_appended = ap;
      st->pipe_eos = eos;
      st->pipe_act = act;
    }
    if (fz == ap) {
      if (lane == 0) plan_none(st, PLAN_STOP);
      return;
    }
    int lo, hi;
    pipe_span(st, fz, &lo, &hi);
    frozen = lo;
    pipe_span(st, ap - 1, &lo, &hi);
    window_end = over ? st->canvas_len + kMaxFwdRows : hi;  // a window too wide fails below
  } else {
    const int bs = st->block_size;
    int bi = st->block_index;
    int rounds = st->rounds_on_block;
    if (st->rounds_cap > 0 && rounds >= st->rounds_cap) {
      bi += bs;
      rounds = 0;
    }
    while (bi < st->gen_len) {
      const int lo = st->prompt_len + bi;
      const int hi = min(lo + bs, st->canvas_len);
      nf = collect_masked(st, x, lo, hi);
      if (nf > 0) {
        frozen = lo;
        window_end = hi;
        break;
      }
      bi += bs;
      rounds = 0;
    }
    __syncwarp();
    if (lane == 0) {
      st->block_index = bi;
      st->rounds_on_block = rounds;
    }
    if (bi >= st->gen_len) {
      if (lane == 0) plan_none(st, PLAN_STOP);
      return;
    }
  }
  if (lane == 0) {
    int pos0 = st->cache_end < frozen ? st->cache_end : frozen;
    // Under dream_ar_shift the first frontier row reads the hidden state of the row before it: that
    // feeder row is forwarded again (its K/V are rewritten from the same final tokens).
    if (st->shift && pos0 > frozen - 1) pos0 = max(frozen - 1, 0);
    const int rows = window_end - pos0;
    if (rows > kMaxFwdRows || nf > kMaxFrontier) {
      st->error = 1;
      plan_none(st, PLAN_STOP);
      return;
    }
    st->action = PLAN_PROCEED;
    st->fwd_pos0 = pos0;
    st->fwd_rows = rows;
    st->kv_len = window_end;
    st->n_frontier = nf;
    for (int i = 0; i < nf; ++i) st->frontier_row[i] = max(st->frontier_pos[i] - st->shift, 0) - pos0;
    st->cache_end = frozen;
  }
}

// One warp. Chooses rows from the device scores, writes the committed tokens into the canvas.
// row_tie (optional): per-row certification bits of the selector (a sampled token within the noise
// rounding bound); those of the committed rows join the step's bits.
__global__ void commit_kernel(DecodeState* st, int* x, const double* conf, const int* token, const int* row_tie,
                              StepTrace* trace) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x;
  __syncwarp();
  const int action = st->action;
  if (action == PLAN_STOP) return;
  if (action == PLAN_SKIP) {
    __syncwarp();
    if (lane == 0) st->step += 1;
    return;
  }
  const int nf = st->n_frontier;
  int k = 0;
  const bool topk = st->policy == POL_BD3_FIXED_QUOTA;
  if (topk) k = st->base + (st->round < st->remainder ? 1 : 0);

  // Each lane owns rows lane and lane + 32.
  unsigned long long chosen = 0ull;
  int tie = 0;
  if (topk) {
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h;
      if (i >= nf) continue;
      const double ci = conf[i];
      int rank = 0;
      for (int j = 0; j < nf; ++j) {
        const double cj = conf[j];
        rank += (cj > ci || (cj == ci && j < i)) ? 1 : 0;
      }
      if (rank < k) chosen |= 1ull << i;
    }
  } else if (st->policy == POL_D2F_PIPELINE) {
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h;
      if (i < nf && conf[i] > st->threshold) chosen |= 1ull << i;
    }
  } else {
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h;
      if (i < nf && conf[i] >= st->threshold) chosen |= 1ull << i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) chosen |= __shfl_xor_sync(0xffffffffu, chosen, o);

  if (lane == 0) {
    const double rel = st->tie_rel;
    if (topk) {
      // k-th largest among chosen and the largest among the rest.
      double kth = INFINITY, next = -INFINITY;
      for (int i = 0; i < nf; ++i) {
        const double c = conf[i];
        if ((chosen >> i) & 1ull) kth = fmin(kth, c);
        else next = fmax(next, c);
      }
      if (k < nf && k > 0) {
        if (kth == next) tie |= TIE_EXACT;
        else if (kth - next <= rel * fabs(kth)) tie |= TIE_NEAR;
      }
    } else if (st->policy == POL_D2F_PIPELINE) {
      const double tau = st->threshold;
      for (int i = 0; i < nf; ++i) {
        if (fabs(conf[i] - tau) <= rel * fabs(tau)) tie |= TIE_NEAR;
      }
      // Per block (frontier rows are in position order, so a block's rows are contiguous): a fully
      // activated block with no row above tau commits its first most-confident row.
      int i = 0;
      while (i < nf) {
        const int b = (st->frontier_pos[i] - st->prompt_len) / st->block_size;
        int end = i;
        unsigned long long rows = 0ull;
        while (end < nf && (st->frontier_pos[end] - st->prompt_len) / st->block_size == b) rows |= 1ull << end++;
        if ((chosen & rows) == 0ull && ((st->pipe_act >> (b - st->pipe_frozen)) & 1ull)) {
          int best = i;
          double b1 = conf[i], b2 = -INFINITY;
          for (int r = i + 1; r < end; ++r) {
            const double c = conf[r];
            if (c > b1) { b2 = b1; b1 = c; best = r; }
            else if (c > b2) { b2 = c; }
          }
          chosen |= 1ull << best;
          if (end - i > 1) {
            if (b1 == b2) tie |= TIE_EXACT;
            else if (b1 - b2 <= rel * fabs(b1)) tie |= TIE_NEAR;
          }
        }
        i = end;
      }
    } else {
      const double tau = st->threshold;
      for (int i = 0; i < nf; ++i) {
        if (fabs(conf[i] - tau) <= rel * fabs(tau)) tie |= TIE_NEAR;
      }
      if (chosen == 0ull && nf > 0) {
        int best = 0;
        double b1 = conf[0], b2 = -INFINITY;
        for (int i = 1; i < nf; ++i) {
          const double c = conf[i];
          if (c > b1) { b2 = b1; b1 = c; best = i; }
          else if (c > b2) { b2 = c; }
        }
        chosen = 1ull << best;
        if (nf > 1) {
          if (b1 == b2) tie |= TIE_EXACT;
          else if (b1 - b2 <= rel * fabs(b1)) tie |= TIE_NEAR;
        }
      }
    }
    int nchosen = 0;
    for (int i = 0; i < nf; ++i) {
      if ((chosen >> i) & 1ull) {
        x[st->frontier_pos[i]] = token[i];
        ++nchosen;
        if (row_tie != nullptr) tie |= row_tie[i] & TIE_NEAR;
      }
    }
    if (trace != nullptr && st->forward_count < st->trace_cap) {
      StepTrace* t = trace + st->forward_count;
      t->step = st->step;
      t->n_frontier = nf;
      t->n_chosen = nchosen;
      t->tie = tie;
      t->chosen_mask = chosen;
      for (int i = 0; i < nf; ++i) {
        t->frontier_pos[i] = st->frontier_pos[i];
        t->token[i] = token[i];
        t->conf[i] = conf[i];
      }
    }
    st->committed_count += nchosen;
    st->iteration_count += 1;
    st->forward_count += 1;
    st->rounds_on_block += 1;
    st->last_tie = tie;
    if (tie & TIE_NEAR) st->near_tie_steps += 1;
    if (tie & TIE_EXACT) st->exact_tie_steps += 1;
    st->step += 1;
  }
}

}  // namespace drt
