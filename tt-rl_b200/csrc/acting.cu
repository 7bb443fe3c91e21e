// Acting heads: the per-lane action choice that follows the acting forward,
// fused into one launch so a whole acting step (frames in, actions out)
// replays from one CUDA graph.
//
// epsilon_greedy_kernel (ttrl/algos/dqn/agent.py:97-119,
// ttrl/algos/mask.py:95-110): greedy = the first maximum of q over the legal
// columns (mask > 0.5; all columns without a mask), then
// action = draws[b] < eps ? alt[b] : greedy. The uniform draws and the
// exploring actions come from the caller's generator, drawn on the host in
// the reference's order, so the choice is the reference's bit for bit.
//
// categorical_sample_kernel (ttrl/algos/ppo/policy.py:36-62): the
// log-softmax of the logits with the operations of the PPO loss kernel (so
// the recorded log-prob and the one the update measures the ratio against are
// the same function), then either the first maximum (deterministic) or the
// inverse-CDF draw against one uniform per lane: probs = exp(logp),
// probs /= sum(probs), cdf = cumulative sum, action = #{j : u > cdf[j]},
// clipped to A-1. One thread per lane.
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

__global__ void epsilon_greedy_kernel(const float* __restrict__ q, const float* __restrict__ mask,
                                      const double* __restrict__ draws,
                                      const int32_t* __restrict__ alt,
                                      const double* __restrict__ eps, int32_t* __restrict__ actions,
                                      int batch, int n_actions) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const float* row = q + static_cast<long long>(b) * n_actions;
  const float* mrow = mask ? mask + static_cast<long long>(b) * n_actions : nullptr;
  int best = 0;
  float bv = -INFINITY;
  bool found = false;
  for (int j = 0; j < n_actions; ++j) {
    if (mrow && !(mrow[j] > 0.5f)) continue;
    const float v = row[j];
    if (!found || v > bv) {
      bv = v;
      best = j;
      found = true;
    }
  }
  actions[b] = (draws != nullptr && eps != nullptr && draws[b] < *eps) ? alt[b] : best;
}

__global__ void categorical_sample_kernel(const float* __restrict__ logits,
                                          const double* __restrict__ uniforms,
                                          int32_t* __restrict__ actions, float* __restrict__ logp,
                                          int batch, int n_actions) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const float* x = logits + static_cast<long long>(b) * n_actions;
  float m = x[0];
  for (int j = 1; j < n_actions; ++j) m = fmaxf(m, x[j]);
  float se = 0.f;
  for (int j = 0; j < n_actions; ++j) se = __fadd_rn(se, expf(__fsub_rn(x[j], m)));
  const float lse = logf(se);
  int act = 0;
  if (uniforms == nullptr) {
    float best = __fsub_rn(__fsub_rn(x[0], m), lse);
    for (int j = 1; j < n_actions; ++j) {
      const float lp = __fsub_rn(__fsub_rn(x[j], m), lse);
      if (lp > best) {
        best = lp;
        act = j;
      }
    }
  } else {
    float total = 0.f;
    for (int j = 0; j < n_actions; ++j)
      total = __fadd_rn(total, expf(__fsub_rn(__fsub_rn(x[j], m), lse)));
    const double u = uniforms[b];
    float cdf = 0.f;
    for (int j = 0; j < n_actions; ++j) {
      const float p = __fdiv_rn(expf(__fsub_rn(__fsub_rn(x[j], m), lse)), total);
      cdf = __fadd_rn(cdf, p);
      if (u > static_cast<double>(cdf)) ++act;
    }
    if (act > n_actions - 1) act = n_actions - 1;
  }
  actions[b] = act;
  if (logp) logp[b] = __fsub_rn(__fsub_rn(x[act], m), lse);
}

int epsilon_greedy(const float* q, const float* mask, const double* draws, const int32_t* alt,
                   const double* eps, int32_t* actions, int batch, int n_actions,
                   cudaStream_t st) {
  if (batch <= 0 || n_actions <= 0)
    return set_error(TTRL_EINVAL, "epsilon_greedy: batch and actions must be > 0");
  if (!q || !actions) return set_error(TTRL_EINVAL, "epsilon_greedy: null pointer");
  if (draws && (!alt || !eps))
    return set_error(TTRL_EINVAL, "epsilon_greedy: draws need exploring actions and eps");
  const cudaError_t le = launch_pdl(epsilon_greedy_kernel, dim3((batch + 127) / 128), dim3(128),
                                    0, st, q, mask, draws, alt, eps, actions, batch, n_actions);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("epsilon_greedy launch", e);
}

int categorical_sample(const float* logits, const double* uniforms, int32_t* actions, float* logp,
                       int batch, int n_actions, cudaStream_t st) {
  if (batch <= 0 || n_actions <= 0)
    return set_error(TTRL_EINVAL, "categorical_sample: batch and actions must be > 0");
  if (!logits || !actions) return set_error(TTRL_EINVAL, "categorical_sample: null pointer");
  const cudaError_t le = launch_pdl(categorical_sample_kernel, dim3((batch + 127) / 128),
                                    dim3(128), 0, st, logits, uniforms, actions, logp, batch,
                                    n_actions);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("categorical_sample launch", e);
}

}  // namespace ttrl

using namespace ttrl;

extern "C" {

int ttrl_epsilon_greedy(const float* q, const float* mask, const double* draws,
                        const int32_t* alt_actions, const double* eps, int32_t* actions, int batch,
                        int n_actions, ttrl_stream_t stream) {
  return epsilon_greedy(q, mask, draws, alt_actions, eps, actions, batch, n_actions,
                        static_cast<cudaStream_t>(stream));
}

int ttrl_categorical_sample(const float* logits, const double* uniforms, int32_t* actions,
                            float* logp, int batch, int n_actions, ttrl_stream_t stream) {
  return categorical_sample(logits, uniforms, actions, logp, batch, n_actions,
                            static_cast<cudaStream_t>(stream));
}

}  // extern "C"
