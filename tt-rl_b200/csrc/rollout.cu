// On-device rollout post-processing for PPO (ttrl/buffers/rollout.py:195-283):
// the GAE-lambda recursion and the advantage normalisation, so a rollout that
// is collected on the device never travels to the host and back before its
// update.
//
// gae_kernel: one thread per environment lane walks t = T-1 .. 0 with the
// reference's float32 operation order (no contraction into fma), so the
// advantages and returns equal the reference's numpy results bit for bit:
//   delta = r[t] + gamma * next * (1 - d[t]) - v[t]
//   gae   = (delta + gamma_lam * (1 - d[t]) * gae) * valid[t]
//   adv[t] = gae; next = v[t];            returns = adv + v
// normalize_kernel: (adv - mean) / (std + 1e-8) over the valid slots (all
// slots when valid is null), the statistics accumulated in double in a fixed
// order inside one block (deterministic), applied in float32.
#include "common.cuh"
#include "internal.h"

namespace ttrl {

__global__ void gae_kernel(const float* __restrict__ rewards, const float* __restrict__ values,
                           const float* __restrict__ dones, const float* __restrict__ valid,
                           const float* __restrict__ last_values, float* __restrict__ adv,
                           float* __restrict__ ret, int steps, int envs, float gamma,
                           float gamma_lam) {
  pdl_trigger();
  pdl_wait();
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= envs) return;
  float next = last_values[e];
  float gae = 0.f;
  for (int t = steps - 1; t >= 0; --t) {
    const long long i = static_cast<long long>(t) * envs + e;
    const float not_done = __fsub_rn(1.f, dones[i]);
    const float v = values[i];
    const float delta =
        __fsub_rn(__fadd_rn(rewards[i], __fmul_rn(__fmul_rn(gamma, next), not_done)), v);
    gae = __fadd_rn(delta, __fmul_rn(__fmul_rn(gamma_lam, not_done), gae));
    if (valid != nullptr) gae = __fmul_rn(gae, valid[i]);
    adv[i] = gae;
    ret[i] = __fadd_rn(gae, v);
    next = v;
  }
}

constexpr int kNormThreads = 1024;

__device__ __forceinline__ double block_sum(double v, double* red) {
  red[threadIdx.x] = v;
  __syncthreads();
  for (int w = kNormThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  const double total = red[0];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kNormThreads) normalize_kernel(const float* __restrict__ adv,
                                                                 const float* __restrict__ valid,
                                                                 float* __restrict__ out,
                                                                 long long n, int* status) {
  pdl_trigger();
  pdl_wait();
  __shared__ double red[kNormThreads];
  double s = 0.0, c = 0.0;
  for (long long i = threadIdx.x; i < n; i += kNormThreads) {
    const bool live = valid == nullptr || valid[i] > 0.f;
    if (live) {
      s += adv[i];
      c += 1.0;
    }
  }
  const double count = block_sum(c, red);
  const double mean = block_sum(s, red) / (count > 0.0 ? count : 1.0);
  double q = 0.0;
  for (long long i = threadIdx.x; i < n; i += kNormThreads) {
    const bool live = valid == nullptr || valid[i] > 0.f;
    if (live) {
      const double d = adv[i] - mean;
      q += d * d;
    }
  }
  const double var = block_sum(q, red) / (count > 0.0 ? count : 1.0);
  if (count <= 0.0) {
    if (threadIdx.x == 0) record_error(status, kErrNoValidSlots);
    return;
  }
  const float mean_f = static_cast<float>(mean);
  const float denom = __fadd_rn(static_cast<float>(sqrt(var)), 1e-8f);
  for (long long i = threadIdx.x; i < n; i += kNormThreads)
    out[i] = __fdiv_rn(__fsub_rn(adv[i], mean_f), denom);
}

int gae(const float* rewards, const float* values, const float* dones, const float* valid,
        const float* last_values, float* adv, float* ret, int steps, int envs, float gamma,
        float gamma_lam, cudaStream_t st) {
  if (steps <= 0 || envs <= 0) return set_error(TTRL_EINVAL, "gae: steps and envs must be > 0");
  if (!rewards || !values || !dones || !last_values || !adv || !ret)
    return set_error(TTRL_EINVAL, "gae: null pointer");
  const int threads = 128;
  const int blocks = (envs + threads - 1) / threads;
  const cudaError_t le = launch_pdl(gae_kernel, dim3(blocks), dim3(threads), 0, st, rewards,
                                    values, dones, valid, last_values, adv, ret, steps, envs,
                                    gamma, gamma_lam);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("gae launch", e);
}

int normalize_advantages(const float* adv, const float* valid, float* out, long long n,
                         int* status, cudaStream_t st) {
  if (n <= 0) return set_error(TTRL_EINVAL, "normalize_advantages: n must be > 0");
  if (!adv || !out) return set_error(TTRL_EINVAL, "normalize_advantages: null pointer");
  const cudaError_t le = launch_pdl(normalize_kernel, dim3(1), dim3(kNormThreads), 0, st, adv,
                                    valid, out, n, status);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("normalize_advantages launch", e);
}

}  // namespace ttrl

using namespace ttrl;

extern "C" {

int ttrl_gae(const float* rewards, const float* values, const float* dones, const float* valid,
             const float* last_values, float* advantages, float* returns, int n_steps,
             int n_envs, float gamma, float gamma_lam, ttrl_stream_t stream) {
  return gae(rewards, values, dones, valid, last_values, advantages, returns, n_steps, n_envs,
             gamma, gamma_lam, static_cast<cudaStream_t>(stream));
}

int ttrl_normalize_advantages(const float* advantages, const float* valid, float* out,
                              long long n, int* status, ttrl_stream_t stream) {
  return normalize_advantages(advantages, valid, out, n, status,
                              static_cast<cudaStream_t>(stream));
}

}  // extern "C"
