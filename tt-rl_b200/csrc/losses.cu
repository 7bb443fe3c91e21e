// Fused loss-and-gradient kernels for DQN and PPO.
//
// Each kernel evaluates the reference's composed loss forward (the same
// sequence of fp32 operations, including the relu-identity spellings of
// min/max/clamp) and writes the gradient of the loss with respect to the
// network outputs in the same launch, so the head of the backward pass is
// one kernel instead of the dozens of elementwise launches the tape issues.
// Reductions use a fixed-shape tree inside one block: deterministic.
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

constexpr int kLossThreads = 1024;

// Fixed-order block sum of one value per thread (all threads get the result).
__device__ float block_sum(float v, float* red) {
  red[threadIdx.x] = v;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  const float s = red[0];
  __syncthreads();
  return s;
}

// ---------------------------------------------------------------- DQN



// ttrl/algos/dqn/losses.py:77-140 (update_loss) with huber from
// ttrl/engine/ops/functional.py:56-69 and the mean of ops/reduce.py:37-41.
__global__ void __launch_bounds__(kLossThreads) dqn_loss_kernel(const __grid_constant__ DqnArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[kLossThreads];
  const int A = a.actions;
  const float inv_b = 1.0f / static_cast<float>(a.batch);
  float err_sum = 0.f, pred_sum = 0.f;
  for (int b = threadIdx.x; b < a.batch; b += blockDim.x) {
    const float* qr = a.q + static_cast<long long>(b) * A;
    const float* oh = a.onehot + static_cast<long long>(b) * A;
    float pred = 0.f;
    for (int j = 0; j < A; ++j) pred = __fadd_rn(pred, __fmul_rn(qr[j], oh[j]));
    // Double-DQN selection: first index of the maximum of the selector,
    // with illegal actions pushed down by (mask - 1) * 1e4 (algos/mask.py:113-121).
    const float* sr = a.q_sel + static_cast<long long>(b) * A;
    int best = 0;
    float bv = 0.f;
    for (int j = 0; j < A; ++j) {
      float v = sr[j];
      if (a.next_mask) {
        const float pen = __fmul_rn(__fsub_rn(a.next_mask[static_cast<long long>(b) * A + j], 1.0f),
                                    1.0e4f);
        v = __fadd_rn(v, pen);
      }
      if (j == 0 || v > bv) {
        bv = v;
        best = j;
      }
    }
    const float next_value = a.q_tgt[static_cast<long long>(b) * A + best];
    const float not_done = __fsub_rn(1.0f, a.dones[b]);
    const float bootstrap = __fmul_rn(__fmul_rn(next_value, not_done), a.discounts[b]);
    const float target = __fadd_rn(a.rewards[b], bootstrap);
    const float e = __fsub_rn(pred, target);
    const float absdiff = fabsf(e);
    const float over = __fsub_rn(absdiff, a.delta);
    const float quad = __fsub_rn(absdiff, relu_f(over));
    const float lin = __fsub_rn(absdiff, quad);
    float err = __fadd_rn(__fmul_rn(__fmul_rn(quad, quad), 0.5f), __fmul_rn(lin, a.delta));
    float g = inv_b;
    if (a.is_weights) {
      err = __fmul_rn(err, a.is_weights[b]);
      g = __fmul_rn(g, a.is_weights[b]);
    }
    err_sum += err;
    pred_sum += pred;
    if (a.td_abs) a.td_abs[b] = absdiff;
    // d huber / d absdiff: delta*g beyond the band, g*quad inside it; then
    // abs' = sign(e) (0 at e == 0).
    const float dabs = over > 0.f ? __fmul_rn(a.delta, g) : __fmul_rn(g, quad);
    const float sgn = e > 0.f ? 1.f : (e < 0.f ? -1.f : 0.f);
    const float de = dabs * sgn;
    float* dqr = a.dq + static_cast<long long>(b) * A;
    for (int j = 0; j < A; ++j) {
      const float v = __fmul_rn(de, oh[j]);
      dqr[j] = a.accumulate ? __fadd_rn(dqr[j], v) : v;
    }
  }
  const float total = block_sum(err_sum, red);
  const float qsum = block_sum(pred_sum, red);
  if (threadIdx.x == 0) {
    a.loss[0] = __fmul_rn(total, inv_b);
    a.mean_q[0] = __fmul_rn(qsum, inv_b);
  }
}

int dqn_loss(const DqnArgs& args, cudaStream_t st) {
  if (args.batch <= 0 || args.actions <= 0) return set_error(TTRL_EINVAL, "dqn_loss: bad extents");
  if (!args.q || !args.q_sel || !args.q_tgt || !args.onehot || !args.rewards || !args.dones ||
      !args.discounts || !args.loss || !args.mean_q || !args.dq)
    return set_error(TTRL_EINVAL, "dqn_loss: null pointer");
  // One thread per sample (a power of two for the reduction tree): the sums
  // are bit-identical to a full-width block's, whose extra levels add zeros.
  int threads = 32;
  while (threads < args.batch && threads < kLossThreads) threads *= 2;
  const cudaError_t le_ = launch_pdl(dqn_loss_kernel, dim3(1), dim3(threads), 0, st, args);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("dqn_loss launch", e);
}

// ---------------------------------------------------------------- PPO



// ttrl/algos/ppo/loss.py:42-83 (objective) with log_softmax / entropy of
// ttrl/engine/ops/functional.py:160-178 and the reducers of loss.py:27-39.
__global__ void __launch_bounds__(kLossThreads) ppo_loss_kernel(const __grid_constant__ PpoArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[kLossThreads];
  const int A = a.num_actions;
  // Denominator of the reducer: B (mean_all) or sum(valid) (masked mean).
  float vsum = 0.f;
  if (a.valid)
    for (int b = threadIdx.x; b < a.batch; b += blockDim.x) vsum += a.valid[b];
  const float denom = a.valid ? block_sum(vsum, red) : static_cast<float>(a.batch);
  const float inv_n = 1.0f / static_cast<float>(a.batch);
  float s_surr = 0.f, s_vmax = 0.f, s_ent = 0.f;
  const float lo = 1.0f - a.clip, hi = 1.0f + a.clip;
  // Per-row loss weights of the reducer (see the gradient derivation below).
  const float g_vl = __fmul_rn(a.vcoef, 0.5f);
  const float g_ent_c = -a.entcoef;
  for (int b = threadIdx.x; b < a.batch; b += blockDim.x) {
    const float* x = a.logits + static_cast<long long>(b) * A;
    float m = x[0];
    for (int j = 1; j < A; ++j) m = fmaxf(m, x[j]);
    float se = 0.f;
    for (int j = 0; j < A; ++j) se = __fadd_rn(se, expf(__fsub_rn(x[j], m)));
    const float lse = logf(se);
    const int act = a.actions[b];
    float nl = 0.f, ent = 0.f;
    for (int j = 0; j < A; ++j) {
      const float lp = __fsub_rn(__fsub_rn(x[j], m), lse);
      if (j == act) nl = lp;
      ent = __fadd_rn(ent, __fmul_rn(expf(lp), lp));
    }
    ent = -ent;
    if (a.new_logp) a.new_logp[b] = nl;
    const float ratio = expf(__fsub_rn(nl, a.old_logp[b]));
    const float A_b = a.adv[b];
    const float s1 = __fmul_rn(ratio, A_b);
    float cpass;
    const float cl = clamp_ref(ratio, lo, hi, cpass);
    const float s2 = __fmul_rn(cl, A_b);
    const float sdiff = __fsub_rn(s1, s2);
    const float surr = __fsub_rn(s1, relu_f(sdiff));
    const float v = a.value[b], ov = a.old_values[b], R = a.returns[b];
    float vpass;
    const float vcl = clamp_ref(__fsub_rn(v, ov), -a.vclip, a.vclip, vpass);
    const float ue = __fsub_rn(v, R);
    const float ce = __fsub_rn(__fadd_rn(ov, vcl), R);
    const float sa = __fmul_rn(ue, ue), sb = __fmul_rn(ce, ce);
    const float bma = __fsub_rn(sb, sa);
    const float vmax = __fadd_rn(sa, relu_f(bma));
    const float w = a.valid ? a.valid[b] : 1.f;
    s_surr += a.valid ? __fmul_rn(surr, w) : surr;
    s_vmax += a.valid ? __fmul_rn(vmax, w) : vmax;
    s_ent += a.valid ? __fmul_rn(ent, w) : ent;

    // Gradient. Per-row reducer weight r = 1/B (mean) or valid/sum(valid).
    const float r = a.valid ? w / denom : inv_n;
    const float g_surr = -r;
    // surrogate = s1 - relu(s1 - s2)
    const float take2 = sdiff > 0.f ? 1.f : 0.f;
    const float ds1 = g_surr * (1.f - take2);
    const float ds2 = g_surr * take2;
    const float dratio = ds1 * A_b + ds2 * A_b * cpass;
    const float dnl = dratio * ratio;  // exp' = exp
    // value: vmax = sa + relu(sb - sa)
    const float gv = g_vl * r;
    const float takeb = bma > 0.f ? 1.f : 0.f;
    const float dsa = gv * (1.f - takeb), dsb = gv * takeb;
    const float dv = 2.f * dsa * ue + 2.f * dsb * ce * vpass;
    a.dvalue[b] = dv;
    // logits: d new_logp and d entropy through the log-softmax.
    const float ge = g_ent_c * r;
    float* dl = a.dlogits + static_cast<long long>(b) * A;
    for (int j = 0; j < A; ++j) {
      const float lp = __fsub_rn(__fsub_rn(x[j], m), lse);
      const float p = expf(lp);
      const float oh = j == act ? 1.f : 0.f;
      dl[j] = dnl * (oh - p) + ge * (-p * (lp + ent));
    }
  }
  const float t_surr = block_sum(s_surr, red);
  const float t_vmax = block_sum(s_vmax, red);
  const float t_ent = block_sum(s_ent, red);
  if (threadIdx.x == 0) {
    const float P = a.valid ? t_surr / denom : __fmul_rn(t_surr, inv_n);
    const float VM = a.valid ? t_vmax / denom : __fmul_rn(t_vmax, inv_n);
    const float EB = a.valid ? t_ent / denom : __fmul_rn(t_ent, inv_n);
    const float policy_loss = -P;
    const float value_loss = __fmul_rn(VM, 0.5f);
    const float loss = __fadd_rn(__fadd_rn(policy_loss, __fmul_rn(value_loss, a.vcoef)),
                                 __fmul_rn(EB, -a.entcoef));
    a.metrics[0] = loss;
    a.metrics[1] = policy_loss;
    a.metrics[2] = value_loss;
    a.metrics[3] = EB;
  }
}

int ppo_loss(const PpoArgs& args, cudaStream_t st) {
  if (args.batch <= 0 || args.num_actions <= 0) return set_error(TTRL_EINVAL, "ppo_loss: bad extents");
  if (!args.logits || !args.value || !args.actions || !args.old_logp || !args.adv ||
      !args.returns || !args.old_values || !args.metrics || !args.dlogits || !args.dvalue)
    return set_error(TTRL_EINVAL, "ppo_loss: null pointer");
  const cudaError_t le_ = launch_pdl(ppo_loss_kernel, dim3(1), dim3(kLossThreads), 0, st, args);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("ppo_loss launch", e);
}

// out[i][:] = src[idx[i]][:] for rows of `row` 4-byte words (float or int32
// payloads alike): the on-device minibatch gather of per-sample fields.
__global__ void gather_rows_kernel(const uint32_t* __restrict__ src, const int32_t* __restrict__ idx,
                                   uint32_t* __restrict__ dst, int n, int row) {
  pdl_trigger();
  pdl_wait();
  const long long total = static_cast<long long>(n) * row;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / row, c = i - r * row;
    dst[i] = src[static_cast<long long>(idx[r]) * row + c];
  }
}

int gather_rows(const void* src, const int32_t* idx, void* dst, int n, int row, cudaStream_t st) {
  if (n <= 0 || row <= 0) return TTRL_OK;
  if (!src || !idx || !dst) return set_error(TTRL_EINVAL, "gather_rows: null pointer");
  const long long total = static_cast<long long>(n) * row;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  const cudaError_t le_ = launch_pdl(gather_rows_kernel, dim3(blocks), dim3(256), 0, st, static_cast<const uint32_t*>(src), idx,
                                            static_cast<uint32_t*>(dst), n, row);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("gather_rows launch", e);
}

// Up to TTRL_GATHER_MAX_JOBS arrays gathered by one index list: blockIdx.y
// picks the array.
struct GatherMultiArgs {
  ttrl_gather_job job[TTRL_GATHER_MAX_JOBS];
  const int32_t* idx;
  int n;
};

__global__ void gather_rows_multi_kernel(const __grid_constant__ GatherMultiArgs a) {
  pdl_trigger();
  pdl_wait();
  const ttrl_gather_job& j = a.job[blockIdx.y];
  const uint32_t* __restrict__ src = static_cast<const uint32_t*>(j.src);
  uint32_t* __restrict__ dst = static_cast<uint32_t*>(j.dst);
  const int row = j.row;
  const long long total = static_cast<long long>(a.n) * row;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / row, c = i - r * row;
    dst[i] = src[static_cast<long long>(a.idx[r]) * row + c];
  }
}

int gather_rows_multi(const ttrl_gather_job* jobs, int count, const int32_t* idx, int n,
                      cudaStream_t st) {
  if (count <= 0 || n <= 0) return TTRL_OK;
  if (count > TTRL_GATHER_MAX_JOBS)
    return set_error(TTRL_EINVAL, "gather_rows_multi: %d arrays (at most %d)", count,
                     TTRL_GATHER_MAX_JOBS);
  if (!jobs || !idx) return set_error(TTRL_EINVAL, "gather_rows_multi: null pointer");
  GatherMultiArgs a;
  std::memset(&a, 0, sizeof(a));
  long long most = 0;
  for (int i = 0; i < count; ++i) {
    if (!jobs[i].src || !jobs[i].dst || jobs[i].row <= 0)
      return set_error(TTRL_EINVAL, "gather_rows_multi: array %d is null or has no columns", i);
    a.job[i] = jobs[i];
    if (jobs[i].row > most) most = jobs[i].row;
  }
  a.idx = idx;
  a.n = n;
  const long long total = most * n;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 4) blocks = 148 * 4;
  const cudaError_t le_ = launch_pdl(gather_rows_multi_kernel, dim3(blocks, count), dim3(256), 0,
                                     st, a);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("gather_rows_multi launch", e);
}

}  // namespace ttrl
