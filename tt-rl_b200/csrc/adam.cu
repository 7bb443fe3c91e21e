// Multi-tensor fused Adam and the deterministic gradient sum of squares.
//
// Adam follows the reference's composed S/V form
// (ttrl/engine/optim/adam.py:93-134): the stored moments are
// S = m/(1-b1) and V = v/(1-b2), and the bias correction folds into two
// scalars (ttrl/engine/optim/scalars.py:13-27). The scalars are computed on
// the device in double precision from a device step counter, so a captured
// CUDA graph replays the correct bias correction at every step.
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

constexpr int kAdamChunk = 8192;   // elements per block
constexpr int kAdamThreads = 256;

struct AdamArgs {
  ttrl_adam_tensor t[TTRL_ADAM_MAX_TENSORS];
  long long chunk_start[TTRL_ADAM_MAX_TENSORS + 1];
  int count;
  int pad0;
  int32_t* steps;
  int32_t* ticket;
  const float* grad_scale;
  const double* lr_device;
  double lr, b1, b2, eps, wd;
};

__global__ void __launch_bounds__(kAdamThreads) adam_kernel(const __grid_constant__ AdamArgs a) {
  // Locate this block's tensor (count <= 64: a linear scan is cheap).
  const long long chunk = blockIdx.x;
  int ti = 0;
  while (ti + 1 < a.count && a.chunk_start[ti + 1] <= chunk) ++ti;
  const ttrl_adam_tensor& T = a.t[ti];
  const long long begin = (chunk - a.chunk_start[ti]) * kAdamChunk;
  const long long end = begin + kAdamChunk < T.numel ? begin + kAdamChunk : T.numel;

  const int step = a.steps[T.step_index] + 1;
  const double bc1 = 1.0 - pow(a.b1, static_cast<double>(step));
  const double bc2 = 1.0 - pow(a.b2, static_cast<double>(step));
  const double c = sqrt((1.0 - a.b2) / bc2);
  const double lr = a.lr_device ? *a.lr_device : a.lr;
  const float alpha_t = static_cast<float>(lr * (1.0 - a.b1) / bc1 / c);
  const float eps_t = static_cast<float>(a.eps / c);
  const float b1 = static_cast<float>(a.b1), b2 = static_cast<float>(a.b2);
  const float wd = static_cast<float>(a.wd);
  const bool scaled = a.grad_scale != nullptr;
  const float gs = scaled ? *a.grad_scale : 1.f;

  // Explicit round-to-nearest intrinsics: no FMA contraction, so each step
  // rounds exactly where the reference's separate device ops round.
  for (long long i = begin + threadIdx.x; i < end; i += blockDim.x) {
    float g = T.grad[i];
    if (scaled) g = __fmul_rn(g, gs);
    const float p = T.param[i];
    if (wd != 0.f) g = __fadd_rn(g, __fmul_rn(wd, p));
    const float sq = __fmul_rn(g, g);
    const float V = __fadd_rn(sq, __fmul_rn(b2, T.v[i]));
    const float S = __fadd_rn(g, __fmul_rn(b1, T.s[i]));
    T.v[i] = V;
    T.s[i] = S;
    float d = __fsqrt_rn(V);
    d = __fadd_rn(d, eps_t);
    d = __fdiv_rn(S, d);
    d = __fmul_rn(d, alpha_t);
    T.param[i] = __fsub_rn(p, d);
  }

  // The last block to finish advances every step counter of this launch,
  // after all blocks have read them.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(reinterpret_cast<unsigned int*>(a.ticket), 1u);
    if (prev == gridDim.x - 1) {
      for (int k = 0; k < a.count; ++k) {
        // Each tensor's counter advances once even if tensors share an index.
        bool seen = false;
        for (int q = 0; q < k; ++q) seen |= a.t[q].step_index == a.t[k].step_index;
        if (!seen) a.steps[a.t[k].step_index] += 1;
      }
      *a.ticket = 0;
      __threadfence();
    }
  }
}

int adam_step(const ttrl_adam_tensor* tensors, int count, int32_t* steps, int32_t* ticket,
              const float* grad_scale, const double* lr_device, double lr, double b1, double b2,
              double eps, double wd, cudaStream_t st) {
  if (count <= 0) return TTRL_OK;
  if (count > TTRL_ADAM_MAX_TENSORS)
    return set_error(TTRL_EINVAL, "adam: %d tensors exceeds the per-call limit %d", count,
                     TTRL_ADAM_MAX_TENSORS);
  if (steps == nullptr || ticket == nullptr)
    return set_error(TTRL_EINVAL, "adam: null step counter or ticket");
  AdamArgs a;
  std::memset(&a, 0, sizeof(a));
  long long chunks = 0;
  for (int i = 0; i < count; ++i) {
    const ttrl_adam_tensor& t = tensors[i];
    if (t.numel <= 0 || !t.param || !t.grad || !t.s || !t.v)
      return set_error(TTRL_EINVAL, "adam: tensor %d is empty or has a null buffer", i);
    a.t[i] = t;
    a.chunk_start[i] = chunks;
    chunks += (t.numel + kAdamChunk - 1) / kAdamChunk;
  }
  a.chunk_start[count] = chunks;
  a.count = count;
  a.steps = steps;
  a.ticket = ticket;
  a.grad_scale = grad_scale;
  a.lr_device = lr_device;
  a.lr = lr;
  a.b1 = b1;
  a.b2 = b2;
  a.eps = eps;
  a.wd = wd;
  adam_kernel<<<static_cast<unsigned>(chunks), kAdamThreads, 0, st>>>(a);
  note_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("adam launch", e);
}

// ------------------------------------------------------ sum of squares

constexpr int kSqChunk = 16384;
constexpr int kSqThreads = 256;

struct SqArgs {
  const float* g[TTRL_ADAM_MAX_TENSORS];
  long long numel[TTRL_ADAM_MAX_TENSORS];
  long long chunk_start[TTRL_ADAM_MAX_TENSORS + 1];
  int count;
  int pad0;
  double* partial;  // one per block
  int32_t* ticket;
  float* out;
  float max_norm;
};

__global__ void __launch_bounds__(kSqThreads) sqnorm_kernel(const __grid_constant__ SqArgs a) {
  __shared__ double red[kSqThreads];
  const long long chunk = blockIdx.x;
  int ti = 0;
  while (ti + 1 < a.count && a.chunk_start[ti + 1] <= chunk) ++ti;
  const long long begin = (chunk - a.chunk_start[ti]) * kSqChunk;
  const long long end = begin + kSqChunk < a.numel[ti] ? begin + kSqChunk : a.numel[ti];
  const float* g = a.g[ti];
  double s = 0.0;
  for (long long i = begin + threadIdx.x; i < end; i += blockDim.x) {
    const double x = g[i];
    s += x * x;
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = kSqThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    a.partial[blockIdx.x] = red[0];
    __threadfence();
    const unsigned int prev = atomicAdd(reinterpret_cast<unsigned int*>(a.ticket), 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      double total = 0.0;
      for (unsigned int b = 0; b < gridDim.x; ++b)
        total += *(volatile double*)(a.partial + b);
      a.out[0] = static_cast<float>(total);
      if (a.max_norm > 0.f) {
        const double norm = sqrt(total);
        const double mx = static_cast<double>(a.max_norm);
        a.out[1] = norm > mx ? static_cast<float>(mx / (norm + 1e-6)) : 1.f;
      }
      *a.ticket = 0;
      __threadfence();
    }
  }
}

size_t sqnorm_ws_bytes(const int64_t* numels, int count) {
  long long chunks = 0;
  for (int i = 0; i < count; ++i) chunks += (numels[i] + kSqChunk - 1) / kSqChunk;
  return 16 + static_cast<size_t>(chunks) * sizeof(double);
}

int grad_sqnorm(const float* const* grads, const int64_t* numels, int count, float* out,
                float max_norm, void* ws, size_t wsb, cudaStream_t st) {
  if (count <= 0) return set_error(TTRL_EINVAL, "grad_sqnorm: no tensors");
  if (count > TTRL_ADAM_MAX_TENSORS)
    return set_error(TTRL_EINVAL, "grad_sqnorm: %d tensors exceeds the limit %d", count,
                     TTRL_ADAM_MAX_TENSORS);
  const size_t need = sqnorm_ws_bytes(numels, count);
  if (ws == nullptr || wsb < need)
    return set_error(TTRL_EWORKSPACE, "grad_sqnorm: needs %zu bytes of workspace, got %zu",
                     need, wsb);
  SqArgs a;
  std::memset(&a, 0, sizeof(a));
  long long chunks = 0;
  for (int i = 0; i < count; ++i) {
    if (numels[i] <= 0 || grads[i] == nullptr)
      return set_error(TTRL_EINVAL, "grad_sqnorm: tensor %d is empty or null", i);
    a.g[i] = grads[i];
    a.numel[i] = numels[i];
    a.chunk_start[i] = chunks;
    chunks += (numels[i] + kSqChunk - 1) / kSqChunk;
  }
  a.chunk_start[count] = chunks;
  a.count = count;
  a.ticket = static_cast<int32_t*>(ws);
  a.partial = reinterpret_cast<double*>(static_cast<char*>(ws) + 16);
  a.out = out;
  a.max_norm = max_norm;
  sqnorm_kernel<<<static_cast<unsigned>(chunks), kSqThreads, 0, st>>>(a);
  note_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("grad_sqnorm launch", e);
}

}  // namespace ttrl
