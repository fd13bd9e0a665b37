// Output decoding on the device: the reference's decode_raw_outputs
// (crates/kata_nn/src/output_postprocess.rs:29-112, run on the host by
// CudaBackend::finish_output, cuda.rs:2510-2600) and, when the caller supplies
// each row's legal-move mask, the evaluator's postprocess_output (:140-330,
// called from eval.rs:675-690).  One CTA per row.
//
// Raw input (the packed forward output, head-major over n rows):
//   policy [n, 6, 362] | value [n, 3] | misc [n, 10] | moremisc [n, 8] | ownership [n, 361]
// Decoded output (head-major over n rows):
//   policy [n, 362] | value [n, 3] | misc [n, 4] | moremisc [n, 2] | ownership [n, 361]
// misc = (score_mean, score_mean_sq, lead, var_time_left), moremisc =
// (shortterm_winloss_error, shortterm_score_error): the NNOutput fields.
//
// Decoding is exact: the symmetry is a permutation and the optimism blend is
// base + (opt - base) * optimism with each f32 operation rounded on its own.
// Post-processing calls CUDA's expf / tanhf (f32) and exp / log / sqrt (f64)
// where the reference calls Rust's f32::exp / tanh and f64::exp / ln / sqrt;
// the policy normaliser sums in index order as the reference does.
#include <stdint.h>

#include "../../include/katab200.h"
#include "kb_internal.h"

namespace kb {
namespace {

constexpr int kSide = 19;
constexpr int kArea = kSide * kSide;  // 361
constexpr int kPolicy = kArea + 1;    // 362: board cells, then pass
constexpr int kThreads = 384;

// copy_outputs_with_symmetry (crates/kata_game/src/symmetry.rs:126-224,
// reverse = true, square board): network cell (r, c) goes to board cell
// (flip_y ? 18 - r : r, flip_x ? 18 - c : c), or under transpose to
// (flip_y ? 18 - c : c, flip_x ? 18 - r : r) — the inverse of the stem's
// input gather.
__device__ __forceinline__ int sym_target(int sym, int r, int c) {
  const int a = (sym & 4) ? c : r;
  const int b = (sym & 4) ? r : c;
  return ((sym & 1) ? kSide - 1 - a : a) * kSide + ((sym & 2) ? kSide - 1 - b : b);
}

__device__ __forceinline__ float blend(float base, float opt, float optimism) {
  // output_postprocess.rs:67-75, no contraction into an FMA.
  return __fadd_rn(base, __fmul_rn(__fsub_rn(opt, base), optimism));
}

__device__ __forceinline__ double softplus(double x) {  // output_postprocess.rs:333-339
  return x > 40.0 ? x : log(1.0 + exp(x));
}

struct DecodeArgs {
  const float* raw;
  const kb_row_params* rows;
  const uint8_t* legal;  // [n, 362] or null: decode only
  kb_postprocess_params pp;
  float* out;
  int n;
};

__global__ void __launch_bounds__(kThreads) decode_rows_kernel(DecodeArgs a) {
  __shared__ float pol[kPolicy];
  __shared__ float red[kThreads / 32];
  __shared__ int cnt[kThreads / 32];
  const int row = blockIdx.x, t = threadIdx.x, n = a.n;
  const kb_row_params rp = a.rows[row];
  const int sym = rp.symmetry & 7;
  const float* raw_pol = a.raw + static_cast<size_t>(row) * 6 * kPolicy;
  const float* raw_val = a.raw + static_cast<size_t>(n) * 6 * kPolicy;
  const float* raw_misc = raw_val + static_cast<size_t>(n) * 3;
  const float* raw_more = raw_misc + static_cast<size_t>(n) * 10;
  const float* raw_own = raw_more + static_cast<size_t>(n) * 8;
  float* out_pol = a.out + static_cast<size_t>(row) * kPolicy;
  float* out_val = a.out + static_cast<size_t>(n) * kPolicy;
  float* out_misc = out_val + static_cast<size_t>(n) * 3;
  float* out_more = out_misc + static_cast<size_t>(n) * 4;
  float* out_own = out_more + static_cast<size_t>(n) * 2;
  const bool post = a.legal != nullptr;

  // decode_raw_outputs: channels 0 and 5 (each with its own pass logit),
  // symmetry undone, blended by the row's optimism.
  if (t < kPolicy) {
    const int dst = t < kArea ? sym_target(sym, t / kSide, t % kSide) : kArea;
    pol[dst] = blend(raw_pol[t], raw_pol[5 * kPolicy + t], rp.policy_optimism);
  }
  if (t < kArea) {
    const int dst = sym_target(sym, t / kSide, t % kSide);
    float v = 0.0f;
    if (rp.include_owner_map) {
      v = raw_own[static_cast<size_t>(row) * kArea + t];
      if (post) {
        // postprocess_output ownership (:313-327): white's perspective, tanh,
        // 0 outside the board.
        if (dst / kSide >= rp.board_y || dst % kSide >= rp.board_x) {
          v = 0.0f;
        } else {
          const float th = tanhf(__fmul_rn(v, a.pp.output_scale_multiplier));
          v = rp.next_player_white ? th : -th;
        }
      }
    }
    out_own[static_cast<size_t>(row) * kArea + dst] = v;
  }
  __syncthreads();

  if (!post) {
    if (t < kPolicy) out_pol[t] = pol[t];
    if (t < 3) out_val[row * 3 + t] = raw_val[row * 3 + t];
    if (t < 4) out_misc[row * 4 + t] = raw_misc[row * 10 + t];
    if (t < 2) out_more[row * 2 + t] = raw_more[row * 8 + t];
    return;
  }

  // postprocess_output, policy (:147-213).
  const kb_postprocess_params& pp = a.pp;
  const float temp = fminf(fmaxf(rp.policy_temperature, 1e-6f), 1e6f);
  const float scaling = __fdiv_rn(pp.output_scale_multiplier, temp);
  const uint8_t* legal = a.legal + static_cast<size_t>(row) * kPolicy;
  const int lane = t & 31, warp = t >> 5;
  float v = -1e30f;
  bool is_legal = false;
  if (t < kPolicy) {
    is_legal = legal[t] != 0;
    if (is_legal) v = __fmul_rn(pol[t], scaling);
  }
  float m = v;
  int c = is_legal ? 1 : 0;
#pragma unroll
  for (int s = 16; s; s >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
    c += __shfl_xor_sync(0xffffffffu, c, s);
  }
  if (lane == 0) {
    red[warp] = m;
    cnt[warp] = c;
  }
  __syncthreads();
  float max_policy = -1e25f;
  int legal_count = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    max_policy = fmaxf(max_policy, red[w]);
    legal_count += cnt[w];
  }
  // Exponentials in parallel; the sum, the pass cap of the passing hacks and
  // the normaliser in index order on one thread, as the reference loops.
  if (t < kPolicy) pol[t] = expf(__fsub_rn(v, max_policy));
  __syncthreads();
  if (t == 0) {
    float sum = 0.0f;
    for (int i = 0; i < kArea; ++i) sum = __fadd_rn(sum, pol[i]);
    float pass = pol[kArea];
    if (rp.passing_hacks) pass = fmaxf(fminf(pass, __fmul_rn(sum, 19.0f)), 1e-20f);  // :173-183
    pol[kArea] = pass;
    red[0] = __fadd_rn(sum, pass);
  }
  if (t == 32) {
    // Value and score (:216-310), f64 as in the reference; every operation
    // rounded on its own (no contraction).
    double vs[3], ms[4], mm[2];
    const double osm = static_cast<double>(pp.output_scale_multiplier);
    if (pp.model_version >= 4) {
#pragma unroll
      for (int i = 0; i < 3; ++i) vs[i] = __dmul_rn(static_cast<double>(raw_val[row * 3 + i]), osm);
#pragma unroll
      for (int i = 0; i < 4; ++i) ms[i] = __dmul_rn(static_cast<double>(raw_misc[row * 10 + i]), osm);
#pragma unroll
      for (int i = 0; i < 2; ++i) mm[i] = __dmul_rn(static_cast<double>(raw_more[row * 8 + i]), osm);
      if (rp.no_result_off) vs[2] = __dsub_rn(vs[2], 100000.0);
      const double mx = fmax(fmax(vs[0], vs[1]), vs[2]);
      double win = exp(__dsub_rn(vs[0], mx)), loss = exp(__dsub_rn(vs[1], mx)), nr = exp(__dsub_rn(vs[2], mx));
      if (rp.no_result_off) nr = 0.0;
      const double psum = __dadd_rn(__dadd_rn(win, loss), nr);
      win = __ddiv_rn(win, psum);
      loss = __ddiv_rn(loss, psum);
      nr = __ddiv_rn(nr, psum);
      double score_mean = __dmul_rn(ms[0], pp.score_mean_multiplier);
      const double score_stdev = __dmul_rn(softplus(ms[1]), pp.score_stdev_multiplier);
      double score_mean_sq = __dadd_rn(__dmul_rn(score_mean, score_mean), __dmul_rn(score_stdev, score_stdev));
      double lead = __dmul_rn(ms[2], pp.lead_multiplier);
      const double var_time = __dmul_rn(softplus(ms[3]), pp.variance_time_multiplier);
      const double keep = __dsub_rn(1.0, nr);
      score_mean = __dmul_rn(score_mean, keep);
      score_mean_sq = __dmul_rn(score_mean_sq, keep);
      lead = __dmul_rn(lead, keep);
      double st_win, st_score;
      if (pp.model_version >= 14) {
        const double s1 = softplus(__dmul_rn(mm[0], 0.5)), s2 = softplus(__dmul_rn(mm[1], 0.5));
        st_win = sqrt(__dmul_rn(__dmul_rn(s1, s1), pp.shortterm_value_error_multiplier));
        st_score = sqrt(__dmul_rn(__dmul_rn(s2, s2), pp.shortterm_score_error_multiplier));
      } else if (pp.model_version >= 10) {
        st_win = sqrt(__dmul_rn(softplus(mm[0]), pp.shortterm_value_error_multiplier));
        st_score = sqrt(__dmul_rn(softplus(mm[1]), pp.shortterm_score_error_multiplier));
      } else {
        st_win = softplus(mm[0]);
        st_score = __dmul_rn(softplus(mm[1]), 10.0);
      }
      const bool white = rp.next_player_white != 0;  // flip to white's perspective (:282-301)
      const float sm = static_cast<float>(score_mean), ld = static_cast<float>(lead);
      out_val[row * 3 + 0] = static_cast<float>(white ? win : loss);
      out_val[row * 3 + 1] = static_cast<float>(white ? loss : win);
      out_val[row * 3 + 2] = static_cast<float>(nr);
      out_misc[row * 4 + 0] = white ? sm : -sm;
      out_misc[row * 4 + 1] = static_cast<float>(score_mean_sq);
      out_misc[row * 4 + 2] = white ? ld : -ld;
      const bool v9 = pp.model_version >= 9;
      out_misc[row * 4 + 3] = v9 ? static_cast<float>(var_time) : -1.0f;
      out_more[row * 2 + 0] = v9 ? static_cast<float>(st_win) : -1.0f;
      out_more[row * 2 + 1] = v9 ? static_cast<float>(st_score) : -1.0f;
    } else {
      for (int i = 0; i < 3; ++i) out_val[row * 3 + i] = raw_val[row * 3 + i];
      for (int i = 0; i < 4; ++i) out_misc[row * 4 + i] = raw_misc[row * 10 + i];
      for (int i = 0; i < 2; ++i) out_more[row * 2 + i] = raw_more[row * 8 + i];
    }
  }
  __syncthreads();
  if (t < kPolicy) {
    const float sum = red[0];
    float p;
    if (!is_legal) p = -1.0f;
    else if (sum <= 0.0f) p = __fdiv_rn(1.0f, static_cast<float>(legal_count > 1 ? legal_count : 1));  // :187-192
    else p = __fdiv_rn(pol[t], sum);
    out_pol[t] = p;
  }
}

int check_rows(const kb_row_params* h_rows, int n) {
  for (int i = 0; i < n; ++i) {
    const kb_row_params& r = h_rows[i];
    if (r.symmetry < 0 || r.symmetry > 7 || !(r.policy_optimism >= 0.0f && r.policy_optimism <= 1.0f) ||
        r.board_x < 1 || r.board_x > kSide || r.board_y < 1 || r.board_y > kSide) {
      set_error("row parameters: need symmetry in 0..7, policy_optimism in [0, 1], board sizes in 1..19");
      return KB_E_INVALID;
    }
  }
  return KB_OK;
}

}  // namespace

kb_postprocess_params default_postprocess_params() {
  // ModelPostProcessParams::default (crates/kata_nn/src/desc.rs:682-695); version 17.
  kb_postprocess_params p;
  p.model_version = 17;
  p.output_scale_multiplier = 1.0f;
  p.td_score_multiplier = 20.0;
  p.score_mean_multiplier = 20.0;
  p.score_stdev_multiplier = 20.0;
  p.lead_multiplier = 20.0;
  p.variance_time_multiplier = 40.0;
  p.shortterm_value_error_multiplier = 0.25;
  p.shortterm_score_error_multiplier = 30.0;
  return p;
}

int check_row_params(const kb_row_params* h_rows, int n) { return check_rows(h_rows, n); }

int decode_rows_launch(int n, const float* raw, const kb_row_params* rows, const uint8_t* legal,
                       const kb_postprocess_params& pp, float* out, cudaStream_t s) {
  if (n <= 0) return KB_OK;
  DecodeArgs a{raw, rows, legal, pp, out, n};
  decode_rows_kernel<<<n, kThreads, 0, s>>>(a);
  return check_cuda(cudaGetLastError(), "output decode launch");
}

}  // namespace kb

using namespace kb;

extern "C" int kb_decode_device(int n, const float* d_raw, const kb_row_params* d_rows, const uint8_t* d_legal,
                                const kb_postprocess_params* pp, float* d_decoded, uintptr_t stream) {
  if (n < 0 || (n > 0 && (!d_raw || !d_rows || !d_decoded))) {
    set_error("kb_decode_device: need n >= 0 and device raw, row and output buffers");
    return KB_E_INVALID;
  }
  const kb_postprocess_params p = pp ? *pp : default_postprocess_params();
  return decode_rows_launch(n, d_raw, d_rows, d_legal, p, d_decoded, reinterpret_cast<cudaStream_t>(stream));
}
