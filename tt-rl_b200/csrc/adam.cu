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

// A block walks chunks of kAdamChunk elements in a grid-stride loop over a
// grid of at most kAdamBlocksPerSM blocks per SM (one wave). Each thread owns
// kAdamQuads float4 quads of a chunk. The operands of the NEXT chunk are
// copied into shared memory asynchronously (cp.async) while the current
// one is computed, so a block keeps its loads in flight through its
// arithmetic instead of alternating between the two; each thread copies and
// later reads only its own shared-memory slots.
constexpr int kAdamThreads = 256;
constexpr int kAdamQuads = 1;
constexpr int kAdamChunk = kAdamThreads * kAdamQuads * 4;  // elements per chunk
constexpr int kAdamBlocksPerSM = 4;

struct AdamArgs {
  ttrl_adam_tensor t[TTRL_ADAM_MAX_TENSORS];
  long long chunk_start[TTRL_ADAM_MAX_TENSORS + 1];
  uint64_t vec_mask;  // bit i: tensor i's four buffers are 16-byte aligned
  int count;
  int pad0;
  int32_t* steps;
  int32_t* ticket;
  const float* grad_scale;
  const double* lr_device;
  const double* bias;     // [bias_steps][2]: (1 - b1^t, c_t) for t = 1.., or null
  long long bias_steps;
  double lr, b1, b2, eps, wd;
};

__device__ __forceinline__ float4 load4(const float* p, long long i, long long end, bool vec) {
  if (vec && i + 3 < end) return *reinterpret_cast<const float4*>(p + i);
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (i < end) v.x = p[i];
  if (i + 1 < end) v.y = p[i + 1];
  if (i + 2 < end) v.z = p[i + 2];
  if (i + 3 < end) v.w = p[i + 3];
  return v;
}

__device__ __forceinline__ void store4(float* p, long long i, long long end, bool vec, float4 v) {
  if (vec && i + 3 < end) {
    *reinterpret_cast<float4*>(p + i) = v;
    return;
  }
  if (i < end) p[i] = v.x;
  if (i + 1 < end) p[i + 1] = v.y;
  if (i + 2 < end) p[i + 2] = v.z;
  if (i + 3 < end) p[i + 3] = v.w;
}

struct AdamScalars {
  float alpha_t, eps_t, b1, b2, wd, gs;
  bool scaled;
};

// One element of the reference's composed tail, rounding where each of its
// separate device ops rounds (explicit _rn intrinsics: no FMA contraction).
__device__ __forceinline__ void adam_elem(const AdamScalars& k, float g, float& p, float& S,
                                          float& V) {
  if (k.scaled) g = __fmul_rn(g, k.gs);
  if (k.wd != 0.f) g = __fadd_rn(g, __fmul_rn(k.wd, p));
  const float sq = __fmul_rn(g, g);
  V = __fadd_rn(sq, __fmul_rn(k.b2, V));
  S = __fadd_rn(g, __fmul_rn(k.b1, S));
  float d = __fsqrt_rn(V);
  d = __fadd_rn(d, k.eps_t);
  d = __fdiv_rn(S, d);
  d = __fmul_rn(d, k.alpha_t);
  p = __fsub_rn(p, d);
}


struct AdamSpan {
  int ti;
  bool vec;
  long long begin, end;
};

// The span of chunk c; `from` is a tensor index at or before c's (a block's
// chunks only move forward, so the scan resumes where the last one ended).
__device__ __forceinline__ AdamSpan adam_span(const AdamArgs& a, long long c, int from) {
  AdamSpan s;
  s.ti = from;
  while (s.ti + 1 < a.count && a.chunk_start[s.ti + 1] <= c) ++s.ti;
  const ttrl_adam_tensor& T = a.t[s.ti];
  s.begin = (c - a.chunk_start[s.ti]) * kAdamChunk;
  s.end = s.begin + kAdamChunk < T.numel ? s.begin + kAdamChunk : T.numel;
  s.vec = (a.vec_mask >> s.ti) & 1ull;
  return s;
}

// Operand order in a stage: gradient, parameter, S, V.
using AdamStage = float4[4][kAdamQuads][kAdamThreads];

// One commit group: this thread's quads of the chunk `s` into `stage`
// (zero-filled past the tensor's end).
__device__ __forceinline__ void adam_prefetch(const AdamArgs& a, const AdamSpan& s,
                                              AdamStage& stage) {
  const ttrl_adam_tensor& T = a.t[s.ti];
  const float* src[4] = {T.grad, T.param, T.s, T.v};
#pragma unroll
  for (int u = 0; u < kAdamQuads; ++u) {
    const long long i = s.begin + (static_cast<long long>(u) * kAdamThreads + threadIdx.x) * 4;
    const long long left = s.end - i;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t dst = smem_u32(&stage[k][u][threadIdx.x]);
      if (s.vec) {
        const uint32_t bytes = left >= 4 ? 16u : (left > 0 ? static_cast<uint32_t>(left) * 4u : 0u);
        cp_async16(dst, bytes ? src[k] + i : src[k], bytes);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const bool in = j < left;
          cp_async4(dst + 4u * j, in ? src[k] + i + j : src[k], in ? 4u : 0u);
        }
      }
    }
  }
  cp_async_commit();
}

__global__ void __launch_bounds__(kAdamThreads, kAdamBlocksPerSM)
    adam_kernel(const __grid_constant__ AdamArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) AdamStage stage[2];
  const long long total = a.chunk_start[a.count];
  long long chunk = blockIdx.x;
  AdamSpan cur{};
  if (chunk < total) {
    cur = adam_span(a, chunk, 0);
    adam_prefetch(a, cur, stage[0]);
  }

  // The bias-correction scalars depend only on a tensor's step: one thread
  // per tensor computes them (double precision) while the first loads are
  // in flight.
  __shared__ AdamScalars ks[TTRL_ADAM_MAX_TENSORS];
  const float gs = a.grad_scale != nullptr ? *a.grad_scale : 1.f;
  for (int q = threadIdx.x; q < a.count; q += blockDim.x) {
    const double lr = a.lr_device ? a.lr_device[a.t[q].lr_index] : a.lr;
    const int step = a.steps[a.t[q].step_index] + 1;
    double bc1, c;
    if (a.bias != nullptr) {
      // Host-computed bias terms: one load instead of two double pow()s.
      const long long t = step < a.bias_steps ? step : a.bias_steps;
      bc1 = a.bias[2 * (t - 1)];
      c = a.bias[2 * (t - 1) + 1];
    } else {
      bc1 = 1.0 - pow(a.b1, static_cast<double>(step));
      const double bc2 = 1.0 - pow(a.b2, static_cast<double>(step));
      c = sqrt((1.0 - a.b2) / bc2);
    }
    AdamScalars k;
    k.alpha_t = static_cast<float>(lr * (1.0 - a.b1) / bc1 / c);
    k.eps_t = static_cast<float>(a.eps / c);
    k.b1 = static_cast<float>(a.b1);
    k.b2 = static_cast<float>(a.b2);
    k.wd = static_cast<float>(a.wd);
    k.scaled = a.grad_scale != nullptr;
    k.gs = gs;
    ks[q] = k;
  }
  __syncthreads();

  int st = 0;
  while (chunk < total) {
    const long long next = chunk + gridDim.x;
    AdamSpan nxt{};
    if (next < total) {
      nxt = adam_span(a, next, cur.ti);
      adam_prefetch(a, nxt, stage[st ^ 1]);
    } else {
      cp_async_commit();  // an empty group: the wait below still means "current chunk in"
    }
    cp_async_wait<1>();
    const AdamScalars k = ks[cur.ti];
    const ttrl_adam_tensor& T = a.t[cur.ti];
#pragma unroll
    for (int u = 0; u < kAdamQuads; ++u) {
      const long long i = cur.begin + (static_cast<long long>(u) * kAdamThreads + threadIdx.x) * 4;
      if (i >= cur.end) continue;
      const float4 g = stage[st][0][u][threadIdx.x];
      float4 p = stage[st][1][u][threadIdx.x];
      float4 S = stage[st][2][u][threadIdx.x];
      float4 V = stage[st][3][u][threadIdx.x];
      adam_elem(k, g.x, p.x, S.x, V.x);
      adam_elem(k, g.y, p.y, S.y, V.y);
      adam_elem(k, g.z, p.z, S.z, V.z);
      adam_elem(k, g.w, p.w, S.w, V.w);
      store4(T.v, i, cur.end, cur.vec, V);
      store4(T.s, i, cur.end, cur.vec, S);
      store4(T.param, i, cur.end, cur.vec, p);
    }
    chunk = next;
    cur = nxt;
    st ^= 1;
  }
  cp_async_wait<0>();

  // The last block to finish advances every step counter of this launch,
  // after all blocks have read them.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(reinterpret_cast<unsigned int*>(a.ticket), 1u);
    if (prev == gridDim.x - 1) {
      for (int q = 0; q < a.count; ++q) {
        // Each tensor's counter advances once even if tensors share an index.
        bool seen = false;
        for (int r = 0; r < q; ++r) seen |= a.t[r].step_index == a.t[q].step_index;
        if (!seen) a.steps[a.t[q].step_index] += 1;
      }
      *a.ticket = 0;
      __threadfence();
    }
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int adam_step(const ttrl_adam_tensor* tensors, int count, int32_t* steps, int32_t* ticket,
              const float* grad_scale, const double* lr_device, double lr, double b1, double b2,
              double eps, double wd, const double* bias, long long bias_steps, cudaStream_t st) {
  if (bias != nullptr && bias_steps < 1)
    return set_error(TTRL_EINVAL, "adam: a bias table needs at least one step");
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
    if (al16(t.param) && al16(t.grad) && al16(t.s) && al16(t.v)) a.vec_mask |= 1ull << i;
    a.chunk_start[i] = chunks;
    chunks += (t.numel + kAdamChunk - 1) / kAdamChunk;
  }
  a.chunk_start[count] = chunks;
  a.count = count;
  a.steps = steps;
  a.ticket = ticket;
  a.grad_scale = grad_scale;
  a.lr_device = lr_device;
  a.bias = bias;
  a.bias_steps = bias_steps;
  a.lr = lr;
  a.b1 = b1;
  a.b2 = b2;
  a.eps = eps;
  a.wd = wd;
  const long long wave = 148LL * kAdamBlocksPerSM;
  const unsigned blocks = static_cast<unsigned>(chunks < wave ? chunks : wave);
  const cudaError_t le_ = launch_pdl(adam_kernel, dim3(blocks), dim3(kAdamThreads), 0, st, a);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("adam launch", e);
}

// ------------------------------------------------------ sum of squares

constexpr int kSqThreads = 256;
constexpr int kSqQuads = 4;
constexpr int kSqChunk = kSqThreads * kSqQuads * 4;

struct SqArgs {
  const float* g[TTRL_ADAM_MAX_TENSORS];
  long long numel[TTRL_ADAM_MAX_TENSORS];
  long long chunk_start[TTRL_ADAM_MAX_TENSORS + 1];
  uint64_t vec_mask;
  int count;
  int pad0;
  double* partial;  // one per block
  int32_t* ticket;
  float* out;
  float max_norm;
};

// Fixed-shape tree sum of kSqThreads doubles in shared memory.
__device__ __forceinline__ double block_sum_fixed(double v, double* red) {
  red[threadIdx.x] = v;
  __syncthreads();
  for (int w = kSqThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  const double total = red[0];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kSqThreads) sqnorm_kernel(const __grid_constant__ SqArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ double red[kSqThreads];
  __shared__ int s_last;
  const long long chunk = blockIdx.x;
  int ti = 0;
  while (ti + 1 < a.count && a.chunk_start[ti + 1] <= chunk) ++ti;
  const long long begin = (chunk - a.chunk_start[ti]) * kSqChunk;
  const long long end = begin + kSqChunk < a.numel[ti] ? begin + kSqChunk : a.numel[ti];
  const bool vec = (a.vec_mask >> ti) & 1ull;
  float4 x[kSqQuads];
#pragma unroll
  for (int u = 0; u < kSqQuads; ++u)
    x[u] = load4(a.g[ti], begin + (static_cast<long long>(u) * kSqThreads + threadIdx.x) * 4,
                 end, vec);
  double s = 0.0;
#pragma unroll
  for (int u = 0; u < kSqQuads; ++u) {
    s += static_cast<double>(x[u].x) * x[u].x;
    s += static_cast<double>(x[u].y) * x[u].y;
    s += static_cast<double>(x[u].z) * x[u].z;
    s += static_cast<double>(x[u].w) * x[u].w;
  }
  const double block_total = block_sum_fixed(s, red);
  if (threadIdx.x == 0) {
    a.partial[blockIdx.x] = block_total;
    __threadfence();
    const unsigned int prev = atomicAdd(reinterpret_cast<unsigned int*>(a.ticket), 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  // The last block sums the per-block partials: every thread takes a fixed
  // strided subset in index order, then the fixed tree, so the total does
  // not depend on which block finished last.
  __threadfence();
  double t = 0.0;
  for (unsigned int b = threadIdx.x; b < gridDim.x; b += kSqThreads) t += __ldcg(a.partial + b);
  const double total = block_sum_fixed(t, red);
  if (threadIdx.x == 0) {
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
    if (al16(grads[i])) a.vec_mask |= 1ull << i;
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
  const cudaError_t le_ = launch_pdl(sqnorm_kernel, dim3(static_cast<unsigned>(chunks)), dim3(kSqThreads), 0, st, a);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("grad_sqnorm launch", e);
}

}  // namespace ttrl
