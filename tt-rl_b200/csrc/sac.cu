// Fused SAC heads: the tanh-squashed Gaussian sample with its log-density,
// its backward, the twin-critic soft-target loss and the actor + temperature
// losses, each one launch.
//
// The reference composes these from generic tape ops (ttrl/algos/gaussian.py,
// ttrl/algos/sac/policy.py, ttrl/algos/sac/losses.py): about a hundred
// elementwise launches per update. Each kernel here evaluates the same
// sequence of fp32 operations -- the relu-identity spellings of min and
// clamp, the stable softplus form of log(1 - tanh(u)^2), the reductions in
// the order the library's own reduce kernel sums -- with explicit _rn
// intrinsics so that no multiply-add is contracted where the composed path
// rounds twice. Loss kernels also write the gradient of the loss with
// respect to their inputs, so the head of the backward pass is free.
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

constexpr int kSampleRows = 128;   // sample forward: one thread per row
constexpr int kSampleBwdThreads = 256;
constexpr int kSacLossThreads = 256;  // the reduction below assumes exactly this
constexpr size_t kSacMaxLossSmem = 200 * 1024;  // per-sample loss terms held on chip

struct SacSampleArgs {
  const float* mean;    // [B][D]
  const float* raw;     // [B][D] log-std before the clamp
  const float* noise;   // [B][D]
  const float* scale;   // [D] half widths of the action box
  const float* centre;  // [D]
  const float* obs;     // [B][obs_dim] or null (obs_dim == 0)
  float* joint;         // [B][obs_dim + D]: obs columns, then the env action
  float* logp;          // [B]
  const float* pack_obs;  // optional second job: [pack_obs | pack_act] rows
  const float* pack_act;
  float* pack_joint;
  int batch, dim, obs_dim;
  float lo, hi, log_det, half_log_2pi_d, log2;
};

// Forward intermediates of one element of the sample, as the composed ops
// round them (ttrl/algos/gaussian.py:55-90, ttrl/algos/sac/policy.py:30-40).
struct SampleElem {
  float ls, pass, std, u, d1, z, v, ex, ad, sp, th;
  float pd;  // z^2 * -0.5 - ls   (one term of the normal log-density sum)
  float c;   // 2 * ((log 2 - u) - softplus(-2u))   (one correction term)
};

__device__ __forceinline__ SampleElem sample_elem(float mean, float raw, float noise, float lo,
                                                  float hi, float log2) {
  SampleElem e;
  e.ls = clamp_ref(raw, lo, hi, e.pass);
  e.std = expf(e.ls);
  e.u = __fadd_rn(mean, __fmul_rn(e.std, noise));
  // normal_logp: z = (u - mean) / exp(log_std); per_dim = z^2 * -0.5 - log_std
  e.d1 = __fsub_rn(e.u, mean);
  e.z = __fdiv_rn(e.d1, e.std);
  e.pd = __fsub_rn(__fmul_rn(__fmul_rn(e.z, e.z), -0.5f), e.ls);
  // log_one_minus_tanh_sq: 2 * ((log 2 - u) - softplus(-2u)), with
  // softplus(x) = relu(x) + log(exp(-|x|) + 1)
  e.v = __fmul_rn(e.u, -2.0f);
  e.ex = expf(__fmul_rn(fabsf(e.v), -1.0f));
  e.ad = __fadd_rn(e.ex, 1.0f);
  e.sp = __fadd_rn(relu_f(e.v), logf(e.ad));
  e.c = __fmul_rn(__fsub_rn(__fsub_rn(log2, e.u), e.sp), 2.0f);
  e.th = tanhf(e.u);
  return e;
}

__global__ void __launch_bounds__(kSampleRows) sac_sample_kernel(const __grid_constant__ SacSampleArgs a) {
  pdl_trigger();
  pdl_wait();
  const int r0 = blockIdx.x * kSampleRows;
  const int rows = a.batch - r0 < kSampleRows ? a.batch - r0 : kSampleRows;
  const int D = a.dim, O = a.obs_dim;
  const long long ld = O + D;
  // The observation columns of the joint rows (and of the packed rows):
  // block-cooperative, reads coalesced.
  for (int i = threadIdx.x; i < rows * O; i += blockDim.x) {
    const int r = i / O, c = i - r * O;
    const long long row = r0 + r;
    a.joint[row * ld + c] = a.obs[row * O + c];
    if (a.pack_joint) a.pack_joint[row * ld + c] = a.pack_obs[row * O + c];
  }
  if (a.pack_joint) {
    for (int i = threadIdx.x; i < rows * D; i += blockDim.x) {
      const int r = i / D, c = i - r * D;
      const long long row = r0 + r;
      a.pack_joint[row * ld + O + c] = a.pack_act[row * D + c];
    }
  }
  if (threadIdx.x >= rows) return;
  const long long b = r0 + threadIdx.x;
  // The two per-row sums over the action dimension run in index order from
  // zero, as the library's reduce kernel sums a short row.
  float normal = 0.f, corr = 0.f;
  for (int d = 0; d < D; ++d) {
    const long long i = b * D + d;
    const SampleElem e = sample_elem(a.mean[i], a.raw[i], a.noise[i], a.lo, a.hi, a.log2);
    normal += e.pd;
    corr += e.c;
    a.joint[b * ld + O + d] = __fadd_rn(__fmul_rn(e.th, a.scale[d]), a.centre[d]);
  }
  normal = __fsub_rn(normal, a.half_log_2pi_d);
  a.logp[b] = __fsub_rn(__fsub_rn(normal, corr), a.log_det);
}

struct SacSampleBwdArgs {
  const float* mean;
  const float* raw;
  const float* noise;
  const float* scale;
  const float* d_action;  // row b, column d at d_action[b * ld + d], or null
  const float* d_logp;    // [B] or null
  float* d_mean;          // [B][D]
  float* d_raw;           // [B][D]
  long long ld;
  int batch, dim, acc_mean, acc_raw;
  float lo, hi, log2;
};

// The backward of the sample: d mean and d raw log-std from the gradient of
// the env action and of the log-density, every product in the order the
// composed ops' backward rules form it.
__global__ void __launch_bounds__(kSampleBwdThreads)
    sac_sample_bwd_kernel(const __grid_constant__ SacSampleBwdArgs a) {
  pdl_trigger();
  pdl_wait();
  const long long n = static_cast<long long>(a.batch) * a.dim;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long b = i / a.dim;
    const int d = static_cast<int>(i - b * a.dim);
    const float mean = a.mean[i], noise = a.noise[i];
    const SampleElem e = sample_elem(mean, a.raw[i], noise, a.lo, a.hi, a.log2);
    float du = 0.f, dmean = 0.f, dls = 0.f;
    if (a.d_action) {
      // action = tanh(u) * scale + centre
      const float dth = __fmul_rn(a.d_action[b * a.ld + d], a.scale[d]);
      du = __fmul_rn(dth, __fsub_rn(1.0f, __fmul_rn(e.th, e.th)));
    }
    if (a.d_logp) {
      const float gl = a.d_logp[b];
      // logp = (sum(per_dim) - c) - sum(corr) - log_det
      // per_dim = z^2 * -0.5 - ls
      dls = -gl;
      const float dz = __fmul_rn(__fmul_rn(gl, -0.5f), __fmul_rn(e.z, 2.0f));
      // z = d1 / std
      const float dd1 = __fdiv_rn(dz, e.std);
      const float dstd_z = __fmul_rn(dz, -__fdiv_rn(e.d1, __fmul_rn(e.std, e.std)));
      // corr term c = 2 * ((log 2 - u) - sp(v)), v = -2u: its gradient is -gl
      const float dt2 = __fmul_rn(-gl, 2.0f);
      const float dsp = -dt2;
      const float dv_relu = e.v > 0.f ? dsp : 0.f;
      const float dnv = __fmul_rn(__fdiv_rn(dsp, e.ad), e.ex);
      const float sgn = e.v > 0.f ? 1.f : (e.v < 0.f ? -1.f : 0.f);
      const float dv = __fadd_rn(dv_relu, __fmul_rn(__fmul_rn(dnv, -1.0f), sgn));
      du = __fadd_rn(du, dd1);
      du = __fadd_rn(du, -dt2);
      du = __fadd_rn(du, __fmul_rn(dv, -2.0f));
      dmean = -dd1;
      dls = __fadd_rn(dls, __fmul_rn(dstd_z, e.std));
    }
    // u = mean + std * noise ; std = exp(ls)
    dmean = __fadd_rn(du, dmean);
    dls = __fadd_rn(dls, __fmul_rn(__fmul_rn(du, noise), e.std));
    const float draw = e.pass != 0.f ? dls : 0.f;
    a.d_mean[i] = a.acc_mean ? __fadd_rn(a.d_mean[i], dmean) : dmean;
    a.d_raw[i] = a.acc_raw ? __fadd_rn(a.d_raw[i], draw) : draw;
  }
}

// The sum ttrl_reduce forms for one row of n values (ops.cu): in index
// order from zero below 1024 values; from 1024 on, 256 strided partial sums
// folded by a fixed tree. Called by all kSacLossThreads threads; every
// thread gets the sum.
__device__ float reduce_order_sum(const float* v, int n, float* red) {
  float acc = 0.f;
  if (n < 1024) {
    if (threadIdx.x == 0) {
      for (int k = 0; k < n; ++k) acc += v[k];
      red[0] = acc;
    }
    __syncthreads();
  } else {
    for (int k = threadIdx.x; k < n; k += blockDim.x) acc += v[k];
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
      if (threadIdx.x < w) red[threadIdx.x] = red[threadIdx.x] + red[threadIdx.x + w];
      __syncthreads();
    }
  }
  const float s = red[0];
  __syncthreads();
  return s;
}

struct SacCriticArgs {
  const float* q[TTRL_SAC_MAX_CRITICS];   // online Q(s, a), [B] each
  const float* qt[TTRL_SAC_MAX_CRITICS];  // target Q(s', a'), [B] each
  float* dq[TTRL_SAC_MAX_CRITICS];        // d loss / d q[i]
  const float* next_logp;
  const float* log_alpha;
  const float* rewards;
  const float* dones;
  const float* discounts;
  const float* weights;  // importance weights or null
  float* loss;
  float* alpha;
  float* target;
  float* td_abs;  // or null
  int n, batch;
  float inv_b, inv_n;
};

// ttrl/algos/sac/losses.py:46-76 (critic_loss) and :30-43 (priority_errors).
__global__ void __launch_bounds__(kSacLossThreads) sac_critic_loss_kernel(const __grid_constant__ SacCriticArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float terms[];  // [n][B] squared (weighted) errors
  __shared__ float red[kSacLossThreads];
  const float alpha = expf(a.log_alpha[0]);
  const float g0 = __fmul_rn(0.5f, a.inv_b);  // d loss / d one squared term
  for (int b = threadIdx.x; b < a.batch; b += blockDim.x) {
    float m = a.qt[0][b];
    for (int i = 1; i < a.n; ++i) m = __fsub_rn(m, relu_f(__fsub_rn(m, a.qt[i][b])));
    const float soft = __fsub_rn(m, __fmul_rn(a.next_logp[b], alpha));
    const float masked = __fmul_rn(soft, __fsub_rn(1.0f, a.dones[b]));
    const float y = __fadd_rn(a.rewards[b], __fmul_rn(masked, a.discounts[b]));
    a.target[b] = y;
    const float w = a.weights ? a.weights[b] : 1.f;
    const float gs = a.weights ? __fmul_rn(g0, w) : g0;
    float abs_sum = 0.f;
    for (int i = 0; i < a.n; ++i) {
      const float e = __fsub_rn(a.q[i][b], y);
      const float sq = __fmul_rn(e, e);
      terms[i * a.batch + b] = a.weights ? __fmul_rn(sq, w) : sq;
      a.dq[i][b] = __fmul_rn(gs, __fmul_rn(e, 2.0f));
      abs_sum = i == 0 ? fabsf(e) : __fadd_rn(abs_sum, fabsf(e));
    }
    if (a.td_abs) a.td_abs[b] = __fmul_rn(abs_sum, a.inv_n);
  }
  __syncthreads();
  float total = 0.f;
  for (int i = 0; i < a.n; ++i) {
    const float mean_i = __fmul_rn(reduce_order_sum(terms + i * a.batch, a.batch, red), a.inv_b);
    total = i == 0 ? mean_i : __fadd_rn(total, mean_i);
  }
  if (threadIdx.x == 0) {
    a.loss[0] = __fmul_rn(total, 0.5f);
    a.alpha[0] = alpha;
  }
}

struct SacActorArgs {
  const float* q[TTRL_SAC_MAX_CRITICS];  // Q_i(s, a~pi), [B] each
  float* dq[TTRL_SAC_MAX_CRITICS];
  const float* logp;
  const float* log_alpha;
  float* loss;
  float* d_logp;
  float* alpha_loss;   // null: no temperature loss
  float* d_log_alpha;
  int n, batch;
  float inv_b, target_entropy;
};

// ttrl/algos/sac/losses.py:79-84 (actor_loss) and :87-95 (alpha_loss); the
// gradients of min over critics follow the relu identity
// min(m, q) = m - relu(m - q): q receives the gradient where m - q > 0.
__global__ void __launch_bounds__(kSacLossThreads) sac_actor_loss_kernel(const __grid_constant__ SacActorArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float terms[];  // [3][B]: actor terms, dual terms, d log alpha terms
  __shared__ float red[kSacLossThreads];
  const float alpha = expf(a.log_alpha[0]);
  const float la = a.log_alpha[0];
  const float dual_g = __fmul_rn(-1.0f, a.inv_b);
  for (int b = threadIdx.x; b < a.batch; b += blockDim.x) {
    float diff[TTRL_SAC_MAX_CRITICS];
    float m = a.q[0][b];
    for (int i = 1; i < a.n; ++i) {
      diff[i] = __fsub_rn(m, a.q[i][b]);
      m = __fsub_rn(m, relu_f(diff[i]));
    }
    const float lp = a.logp[b];
    terms[b] = __fsub_rn(__fmul_rn(lp, alpha), m);
    a.d_logp[b] = __fmul_rn(a.inv_b, alpha);
    float gm = -a.inv_b;
    for (int i = a.n - 1; i >= 1; --i) {
      const float r = diff[i] > 0.f ? -gm : 0.f;
      a.dq[i][b] = -r;
      gm = __fadd_rn(gm, r);
    }
    a.dq[0][b] = gm;
    if (a.alpha_loss) {
      const float t = __fadd_rn(lp, a.target_entropy);
      terms[a.batch + b] = __fmul_rn(la, t);
      terms[2 * a.batch + b] = __fmul_rn(dual_g, t);
    }
  }
  __syncthreads();
  const float loss = __fmul_rn(reduce_order_sum(terms, a.batch, red), a.inv_b);
  float dual = 0.f, dla = 0.f;
  if (a.alpha_loss) {
    dual = __fmul_rn(__fmul_rn(reduce_order_sum(terms + a.batch, a.batch, red), a.inv_b), -1.0f);
    dla = reduce_order_sum(terms + 2 * a.batch, a.batch, red);
  }
  if (threadIdx.x == 0) {
    a.loss[0] = loss;
    if (a.alpha_loss) {
      a.alpha_loss[0] = dual;
      a.d_log_alpha[0] = dla;
    }
  }
}

namespace {

int launched(const char* what, cudaError_t le) {
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error(what, e);
}

// Dynamic shared memory of a loss kernel: `arrays` float arrays of `batch`.
int loss_smem(const void* kernel, int arrays, int batch, size_t* bytes) {
  *bytes = static_cast<size_t>(arrays) * batch * sizeof(float);
  if (*bytes > kSacMaxLossSmem)
    return set_error(TTRL_EUNSUPPORTED,
                     "sac loss: batch %d needs %zu bytes of shared memory, the kernel holds at "
                     "most %zu", batch, *bytes, static_cast<size_t>(kSacMaxLossSmem));
  if (*bytes > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(*bytes));
    if (e != cudaSuccess) return set_cuda_error("sac loss: shared-memory limit", e);
  }
  return TTRL_OK;
}

}  // namespace

int sac_sample(const SacSampleArgs& a, cudaStream_t st) {
  if (a.batch <= 0 || a.dim <= 0 || a.obs_dim < 0)
    return set_error(TTRL_EINVAL, "sac_sample: bad extents batch=%d dim=%d obs_dim=%d", a.batch,
                     a.dim, a.obs_dim);
  if (!a.mean || !a.raw || !a.noise || !a.scale || !a.centre || !a.joint || !a.logp)
    return set_error(TTRL_EINVAL, "sac_sample: null pointer");
  if (a.obs_dim > 0 && !a.obs) return set_error(TTRL_EINVAL, "sac_sample: obs_dim > 0, obs null");
  if (a.pack_joint && (a.obs_dim == 0 || !a.pack_obs || !a.pack_act))
    return set_error(TTRL_EINVAL, "sac_sample: packing needs obs columns and both sources");
  if (!(a.lo < a.hi)) return set_error(TTRL_EINVAL, "sac_sample: log_std_min >= log_std_max");
  const int blocks = (a.batch + kSampleRows - 1) / kSampleRows;
  return launched("sac_sample launch",
                  launch_pdl(sac_sample_kernel, dim3(blocks), dim3(kSampleRows), 0, st, a));
}

int sac_sample_backward(const SacSampleBwdArgs& a, cudaStream_t st) {
  if (a.batch <= 0 || a.dim <= 0) return set_error(TTRL_EINVAL, "sac_sample_backward: bad extents");
  if (!a.mean || !a.raw || !a.noise || !a.scale || !a.d_mean || !a.d_raw)
    return set_error(TTRL_EINVAL, "sac_sample_backward: null pointer");
  if (a.d_action && a.ld < a.dim)
    return set_error(TTRL_EINVAL, "sac_sample_backward: row stride %lld below the action width %d",
                     a.ld, a.dim);
  const long long n = static_cast<long long>(a.batch) * a.dim;
  long long blocks = (n + kSampleBwdThreads - 1) / kSampleBwdThreads;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launched("sac_sample_backward launch",
                  launch_pdl(sac_sample_bwd_kernel, dim3(static_cast<unsigned>(blocks)),
                             dim3(kSampleBwdThreads), 0, st, a));
}

int sac_critic_loss(const SacCriticArgs& a, cudaStream_t st) {
  if (a.batch <= 0 || a.n < 1 || a.n > TTRL_SAC_MAX_CRITICS)
    return set_error(TTRL_EINVAL, "sac_critic_loss: batch %d, %d critics (1..%d)", a.batch, a.n,
                     TTRL_SAC_MAX_CRITICS);
  for (int i = 0; i < a.n; ++i)
    if (!a.q[i] || !a.qt[i] || !a.dq[i]) return set_error(TTRL_EINVAL, "sac_critic_loss: null critic");
  if (!a.next_logp || !a.log_alpha || !a.rewards || !a.dones || !a.discounts || !a.loss ||
      !a.alpha || !a.target)
    return set_error(TTRL_EINVAL, "sac_critic_loss: null pointer");
  size_t smem = 0;
  const int rc = loss_smem(reinterpret_cast<const void*>(sac_critic_loss_kernel), a.n, a.batch, &smem);
  if (rc) return rc;
  return launched("sac_critic_loss launch",
                  launch_pdl(sac_critic_loss_kernel, dim3(1), dim3(kSacLossThreads), smem, st, a));
}

int sac_actor_loss(const SacActorArgs& a, cudaStream_t st) {
  if (a.batch <= 0 || a.n < 1 || a.n > TTRL_SAC_MAX_CRITICS)
    return set_error(TTRL_EINVAL, "sac_actor_loss: batch %d, %d critics (1..%d)", a.batch, a.n,
                     TTRL_SAC_MAX_CRITICS);
  for (int i = 0; i < a.n; ++i)
    if (!a.q[i] || !a.dq[i]) return set_error(TTRL_EINVAL, "sac_actor_loss: null critic");
  if (!a.logp || !a.log_alpha || !a.loss || !a.d_logp)
    return set_error(TTRL_EINVAL, "sac_actor_loss: null pointer");
  if (a.alpha_loss && !a.d_log_alpha)
    return set_error(TTRL_EINVAL, "sac_actor_loss: temperature loss without its gradient");
  size_t smem = 0;
  const int rc = loss_smem(reinterpret_cast<const void*>(sac_actor_loss_kernel), 3, a.batch, &smem);
  if (rc) return rc;
  return launched("sac_actor_loss launch",
                  launch_pdl(sac_actor_loss_kernel, dim3(1), dim3(kSacLossThreads), smem, st, a));
}

}  // namespace ttrl

using namespace ttrl;

extern "C" {

int ttrl_sac_sample(const float* mean, const float* log_std_raw, const float* noise,
                    const float* scale, const float* centre, const float* obs, float* joint,
                    float* logp, int batch, int action_dim, int obs_dim, float log_std_min,
                    float log_std_max, float log_det, const float* pack_obs,
                    const float* pack_act, float* pack_joint, ttrl_stream_t stream) {
  SacSampleArgs a;
  std::memset(&a, 0, sizeof(a));
  a.mean = mean, a.raw = log_std_raw, a.noise = noise, a.scale = scale, a.centre = centre;
  a.obs = obs, a.joint = joint, a.logp = logp;
  a.pack_obs = pack_obs, a.pack_act = pack_act, a.pack_joint = pack_joint;
  a.batch = batch, a.dim = action_dim, a.obs_dim = obs_dim;
  a.lo = log_std_min, a.hi = log_std_max, a.log_det = log_det;
  // The two scalars the composed path passes as fp32 constants.
  a.half_log_2pi_d = static_cast<float>(0.5 * action_dim * std::log(2.0 * M_PI));
  a.log2 = static_cast<float>(std::log(2.0));
  return sac_sample(a, static_cast<cudaStream_t>(stream));
}

int ttrl_sac_sample_backward(const float* mean, const float* log_std_raw, const float* noise,
                             const float* scale, const float* d_action, int64_t d_action_ld,
                             const float* d_logp, float* d_mean, float* d_log_std_raw,
                             int accumulate_mean, int accumulate_log_std, int batch,
                             int action_dim, float log_std_min, float log_std_max,
                             ttrl_stream_t stream) {
  SacSampleBwdArgs a;
  std::memset(&a, 0, sizeof(a));
  a.mean = mean, a.raw = log_std_raw, a.noise = noise, a.scale = scale;
  a.d_action = d_action, a.d_logp = d_logp, a.d_mean = d_mean, a.d_raw = d_log_std_raw;
  a.ld = d_action_ld, a.batch = batch, a.dim = action_dim;
  a.acc_mean = accumulate_mean, a.acc_raw = accumulate_log_std;
  a.lo = log_std_min, a.hi = log_std_max;
  a.log2 = static_cast<float>(std::log(2.0));
  return sac_sample_backward(a, static_cast<cudaStream_t>(stream));
}

int ttrl_sac_critic_loss(const float* const* q, const float* const* q_target, int n_critics,
                         const float* next_logp, const float* log_alpha, const float* rewards,
                         const float* dones, const float* discounts, const float* is_weights,
                         float* loss, float* alpha, float* target, float* const* dq,
                         float* td_abs, int batch, ttrl_stream_t stream) {
  if (!q || !q_target || !dq) return set_error(TTRL_EINVAL, "sac_critic_loss: null critic list");
  if (n_critics < 1 || n_critics > TTRL_SAC_MAX_CRITICS)
    return set_error(TTRL_EINVAL, "sac_critic_loss: %d critics (1..%d)", n_critics,
                     TTRL_SAC_MAX_CRITICS);
  SacCriticArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int i = 0; i < n_critics; ++i) a.q[i] = q[i], a.qt[i] = q_target[i], a.dq[i] = dq[i];
  a.next_logp = next_logp, a.log_alpha = log_alpha, a.rewards = rewards, a.dones = dones;
  a.discounts = discounts, a.weights = is_weights;
  a.loss = loss, a.alpha = alpha, a.target = target, a.td_abs = td_abs;
  a.n = n_critics, a.batch = batch;
  a.inv_b = batch > 0 ? static_cast<float>(1.0 / batch) : 0.f;
  a.inv_n = static_cast<float>(1.0 / n_critics);
  return sac_critic_loss(a, static_cast<cudaStream_t>(stream));
}

int ttrl_sac_actor_loss(const float* const* q, int n_critics, const float* logp,
                        const float* log_alpha, float target_entropy, float* loss,
                        float* const* dq, float* d_logp, float* alpha_loss,
                        float* d_log_alpha, int batch, ttrl_stream_t stream) {
  if (!q || !dq) return set_error(TTRL_EINVAL, "sac_actor_loss: null critic list");
  if (n_critics < 1 || n_critics > TTRL_SAC_MAX_CRITICS)
    return set_error(TTRL_EINVAL, "sac_actor_loss: %d critics (1..%d)", n_critics,
                     TTRL_SAC_MAX_CRITICS);
  SacActorArgs a;
  std::memset(&a, 0, sizeof(a));
  for (int i = 0; i < n_critics; ++i) a.q[i] = q[i], a.dq[i] = dq[i];
  a.logp = logp, a.log_alpha = log_alpha, a.loss = loss, a.d_logp = d_logp;
  a.alpha_loss = alpha_loss, a.d_log_alpha = d_log_alpha;
  a.n = n_critics, a.batch = batch;
  a.inv_b = batch > 0 ? static_cast<float>(1.0 / batch) : 0.f;
  a.target_entropy = target_entropy;
  return sac_actor_loss(a, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
