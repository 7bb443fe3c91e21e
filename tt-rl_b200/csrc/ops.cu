// Elementwise, reduction and strided-copy kernels behind the generic tape
// ops (ttrl/engine/ops/{elementwise,unary,select,reduce,shape}.py). Each op
// is one launch; reductions are sequential per output element (or a fixed
// tree inside one block), so results are deterministic.
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

struct EwArgs {
  int op;
  int ndim;
  float scalar;
  int pad0;
  const float* a;
  const float* b;
  float* out;
  int64_t n;
  int64_t shape[4];
  int64_t as[4];
  int64_t bs[4];
};

__device__ __forceinline__ float ew_apply(int op, float x, float y, float s) {
  switch (op) {
    case TTRL_EW_ADD: return x + y;
    case TTRL_EW_SUB: return x - y;
    case TTRL_EW_MUL: return x * y;
    case TTRL_EW_DIV: return x / y;
    case TTRL_EW_ADD_S: return x + s;
    case TTRL_EW_SUB_S: return x - s;
    case TTRL_EW_RSUB_S: return s - x;
    case TTRL_EW_MUL_S: return x * s;
    case TTRL_EW_DIV_S: return x / s;
    case TTRL_EW_RELU: return x > 0.f ? x : 0.f;
    case TTRL_EW_RELU_BW: return y > 0.f ? x : 0.f;  // x = grad, y = forward input
    case TTRL_EW_ABS: return fabsf(x);
    case TTRL_EW_SIGN: return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
    case TTRL_EW_NEG: return -x;
    case TTRL_EW_EXP: return expf(x);
    case TTRL_EW_LOG: return logf(x);
    case TTRL_EW_TANH: return tanhf(x);
    case TTRL_EW_SIGMOID: return 1.f / (1.f + expf(-x));
    case TTRL_EW_SQRT: return sqrtf(x);
    case TTRL_EW_SQUARE: return x * x;
    case TTRL_EW_EQZ: return x == 0.f ? 1.f : 0.f;
    case TTRL_EW_FILL: return s;
    case TTRL_EW_COPY: return x;
    case TTRL_EW_GT_S: return x > s ? 1.f : 0.f;
    case TTRL_EW_EQ: return x == y ? 1.f : 0.f;
    default: return 0.f;
  }
}

__global__ void ew_kernel(const __grid_constant__ EwArgs a) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < a.n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t rem = i, ao = 0, bo = 0;
#pragma unroll
    for (int d = 3; d >= 0; --d) {
      if (d < a.ndim) {
        const int64_t idx = rem % a.shape[d];
        rem /= a.shape[d];
        ao += idx * a.as[d];
        bo += idx * a.bs[d];
      }
    }
    const float x = a.a ? a.a[ao] : 0.f;
    const float y = a.b ? a.b[bo] : 0.f;
    a.out[i] = ew_apply(a.op, x, y, a.scalar);
  }
}

int ew(int op, const float* x, const int64_t* xs, const float* y, const int64_t* ys, float* out,
       const int64_t* shape, int ndim, float scalar, cudaStream_t st) {
  if (ndim < 1 || ndim > 4) return set_error(TTRL_EINVAL, "ew: rank %d outside [1, 4]", ndim);
  if (out == nullptr) return set_error(TTRL_EINVAL, "ew: null output");
  EwArgs a;
  std::memset(&a, 0, sizeof(a));
  a.op = op;
  a.ndim = ndim;
  a.scalar = scalar;
  a.a = x;
  a.b = y;
  a.out = out;
  int64_t n = 1;
  for (int d = 0; d < ndim; ++d) {
    if (shape[d] < 0) return set_error(TTRL_EINVAL, "ew: negative extent");
    a.shape[d] = shape[d];
    a.as[d] = xs ? xs[d] : 0;
    a.bs[d] = ys ? ys[d] : 0;
    n *= shape[d];
  }
  a.n = n;
  if (n == 0) return TTRL_OK;
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  const cudaError_t le_ = launch_pdl(ew_kernel, dim3(blocks), dim3(256), 0, st, a);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("ew launch", e);
}

// ------------------------------------------------------------ reductions

// in viewed as [outer][n][inner]; out [outer][inner].
__global__ void reduce_thread_kernel(int op, const float* __restrict__ in, float* __restrict__ out,
                                     int64_t outer, int64_t n, int64_t inner) {
  pdl_trigger();
  pdl_wait();
  const int64_t total = outer * inner;
  for (int64_t o = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; o < total;
       o += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i0 = o / inner, j = o - i0 * inner;
    const float* p = in + i0 * n * inner + j;
    if (op == TTRL_RED_SUM) {
      float s = 0.f;
      for (int64_t k = 0; k < n; ++k) s += p[k * inner];
      out[o] = s;
    } else {
      float best = p[0];
      int64_t arg = 0;
      for (int64_t k = 1; k < n; ++k) {
        const float v = p[k * inner];
        if (v > best) {
          best = v;
          arg = k;
        }
      }
      out[o] = op == TTRL_RED_MAX ? best : static_cast<float>(arg);
    }
  }
}

// One block per output element, fixed-shape tree: for long reductions.
__global__ void reduce_block_kernel(int op, const float* __restrict__ in, float* __restrict__ out,
                                    int64_t n, int64_t inner) {
  pdl_trigger();
  pdl_wait();
  __shared__ float vals[256];
  __shared__ int64_t args[256];
  const int64_t o = blockIdx.x;
  const int64_t i0 = o / inner, j = o - i0 * inner;
  const float* p = in + i0 * n * inner + j;
  float acc = op == TTRL_RED_SUM ? 0.f : -INFINITY;
  int64_t arg = n;  // argmax: smallest index among maxima
  for (int64_t k = threadIdx.x; k < n; k += blockDim.x) {
    const float v = p[k * inner];
    if (op == TTRL_RED_SUM) {
      acc += v;
    } else if (v > acc || arg == n) {
      if (!(v <= acc) || arg == n) {
        acc = v;
        arg = k;
      }
    }
  }
  vals[threadIdx.x] = acc;
  args[threadIdx.x] = arg;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      const float a = vals[threadIdx.x], b = vals[threadIdx.x + w];
      if (op == TTRL_RED_SUM) {
        vals[threadIdx.x] = a + b;
      } else {
        const int64_t ia = args[threadIdx.x], ib = args[threadIdx.x + w];
        const bool take_b = (ib != n) && (ia == n || b > a || (b == a && ib < ia));
        if (take_b) {
          vals[threadIdx.x] = b;
          args[threadIdx.x] = ib;
        }
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0)
    out[o] = op == TTRL_RED_ARGMAX ? static_cast<float>(args[0]) : vals[0];
}

int reduce(int op, const float* in, float* out, int64_t outer, int64_t n, int64_t inner,
           cudaStream_t st) {
  if (in == nullptr || out == nullptr) return set_error(TTRL_EINVAL, "reduce: null pointer");
  if (outer <= 0 || n <= 0 || inner <= 0) return set_error(TTRL_EINVAL, "reduce: empty extent");
  const int64_t total = outer * inner;
  cudaError_t le_;
  if (total < 512 && n >= 1024) {
    le_ = launch_pdl(reduce_block_kernel, dim3(static_cast<unsigned>(total)), dim3(256), 0, st,
                     op, in, out, n, inner);
    note_launch();
  } else {
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > 148 * 8) blocks = 148 * 8;
    le_ = launch_pdl(reduce_thread_kernel, dim3(blocks), dim3(256), 0, st, op, in, out, outer, n, inner);
    note_launch();
  }
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("reduce launch", e);
}

// ---------------------------------------------------------- strided copy

__global__ void copy_strided_kernel(const __grid_constant__ EwArgs a) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < a.n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t rem = i, so = 0, dof = 0;
#pragma unroll
    for (int d = 3; d >= 0; --d) {
      if (d < a.ndim) {
        const int64_t idx = rem % a.shape[d];
        rem /= a.shape[d];
        so += idx * a.as[d];
        dof += idx * a.bs[d];
      }
    }
    float v = a.a[so];
    if (a.op) v += a.out[dof];
    a.out[dof] = v;
  }
}

int copy_strided(float* dst, const int64_t* ds, const float* src, const int64_t* ss,
                 const int64_t* shape, int ndim, int accumulate, cudaStream_t st) {
  if (ndim < 1 || ndim > 4) return set_error(TTRL_EINVAL, "copy: rank %d outside [1, 4]", ndim);
  if (dst == nullptr || src == nullptr) return set_error(TTRL_EINVAL, "copy: null pointer");
  EwArgs a;
  std::memset(&a, 0, sizeof(a));
  a.op = accumulate;
  a.ndim = ndim;
  a.a = src;
  a.out = dst;
  int64_t n = 1;
  for (int d = 0; d < ndim; ++d) {
    a.shape[d] = shape[d];
    a.as[d] = ss[d];
    a.bs[d] = ds[d];
    n *= shape[d];
  }
  a.n = n;
  if (n == 0) return TTRL_OK;
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  const cudaError_t le_ = launch_pdl(copy_strided_kernel, dim3(blocks), dim3(256), 0, st, a);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("copy launch", e);
}

// ------------------------------------------------------ Polyak / average

__global__ void axpby_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n,
                             float keep, float take) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    // Order of ttrl/algos/sac/targets.py:55-61: add(mul(dst, 1-tau), mul(src, tau)).
    const float a = dst[i] * keep;
    const float b = src[i] * take;
    dst[i] = a + b;
  }
}

int polyak(float* dst, const float* src, int64_t n, float tau, cudaStream_t st) {
  if (n <= 0) return TTRL_OK;
  if (dst == nullptr || src == nullptr) return set_error(TTRL_EINVAL, "polyak: null pointer");
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  const cudaError_t le_ = launch_pdl(axpby_kernel, dim3(blocks), dim3(256), 0, st, dst, src, n, 1.0f - tau, tau);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("polyak launch", e);
}

// ------------------------------------------------- multi-tensor blend/copy

// One launch over a list of (dst, src, n) pairs: the DQN hard target copy
// (dst = src, bit for bit) or the Polyak blend (dst = (1-tau) dst + tau src)
// of every parameter of a network. The pairs are cut into tiles of
// kBlendTile elements; a block takes tiles in a grid-stride loop and finds
// each tile's pair among the <= kBlendMax prefix sums.
constexpr int kBlendMax = 48;
constexpr int kBlendTile = 4096;

struct BlendArgs {
  int count;
  int mode;
  float keep, take;
  float* dst[kBlendMax];
  const float* src[kBlendMax];
  int64_t n[kBlendMax];
  int64_t first_tile[kBlendMax + 1];
};

__global__ void __launch_bounds__(256) blend_kernel(const __grid_constant__ BlendArgs a) {
  pdl_trigger();
  pdl_wait();
  const int64_t tiles = a.first_tile[a.count];
  int t = 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    while (a.first_tile[t + 1] <= tile) ++t;
    const int64_t base = (tile - a.first_tile[t]) * kBlendTile;
    const int64_t left = a.n[t] - base;
    const int64_t len = left < kBlendTile ? left : kBlendTile;
    float* __restrict__ d = a.dst[t] + base;
    const float* __restrict__ s = a.src[t] + base;
    const bool vec = ((reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(s)) & 15) == 0;
    const int64_t nvec = vec ? len / 4 : 0;
    for (int64_t i = threadIdx.x; i < nvec; i += blockDim.x) {
      const float4 x = reinterpret_cast<const float4*>(s)[i];
      float4 y;
      if (a.mode == TTRL_BLEND_COPY) {
        y = x;
      } else {
        // Order of ttrl/algos/sac/targets.py:55-61: add(mul(dst, 1-tau),
        // mul(src, tau)), each rounded on its own (no fused multiply-add).
        const float4 o = reinterpret_cast<const float4*>(d)[i];
        y.x = __fadd_rn(__fmul_rn(o.x, a.keep), __fmul_rn(x.x, a.take));
        y.y = __fadd_rn(__fmul_rn(o.y, a.keep), __fmul_rn(x.y, a.take));
        y.z = __fadd_rn(__fmul_rn(o.z, a.keep), __fmul_rn(x.z, a.take));
        y.w = __fadd_rn(__fmul_rn(o.w, a.keep), __fmul_rn(x.w, a.take));
      }
      reinterpret_cast<float4*>(d)[i] = y;
    }
    for (int64_t i = nvec * 4 + threadIdx.x; i < len; i += blockDim.x) {
      if (a.mode == TTRL_BLEND_COPY) {
        d[i] = s[i];
      } else {
        d[i] = __fadd_rn(__fmul_rn(d[i], a.keep), __fmul_rn(s[i], a.take));
      }
    }
  }
}

int blend_multi(const ttrl_blend_pair* pairs, int count, int mode, float tau, cudaStream_t st) {
  if (count < 0 || (count > 0 && pairs == nullptr))
    return set_error(TTRL_EINVAL, "blend_multi: bad pair list");
  if (mode != TTRL_BLEND_COPY && mode != TTRL_BLEND_POLYAK)
    return set_error(TTRL_EINVAL, "blend_multi: unknown mode %d", mode);
  for (int start = 0; start < count; start += kBlendMax) {
    BlendArgs a;
    std::memset(&a, 0, sizeof(a));
    a.mode = mode;
    a.keep = 1.0f - tau;
    a.take = tau;
    int64_t tiles = 0;
    for (int i = start; i < count && a.count < kBlendMax; ++i) {
      const ttrl_blend_pair& p = pairs[i];
      if (p.n < 0 || (p.n > 0 && (p.dst == nullptr || p.src == nullptr)))
        return set_error(TTRL_EINVAL, "blend_multi: pair %d has a null pointer or n < 0", i);
      if (p.n == 0) continue;
      a.dst[a.count] = p.dst;
      a.src[a.count] = p.src;
      a.n[a.count] = p.n;
      a.first_tile[a.count] = tiles;
      tiles += (p.n + kBlendTile - 1) / kBlendTile;
      ++a.count;
    }
    if (a.count == 0) continue;
    a.first_tile[a.count] = tiles;
    int blocks = static_cast<int>(tiles < 148 * 4 ? tiles : 148 * 4);
    const cudaError_t le = launch_pdl(blend_kernel, dim3(blocks), dim3(256), 0, st, a);
    note_launch();
    const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("blend_multi launch", e);
  }
  return TTRL_OK;
}

// ------------------------------------------------------- bounded-wait check

// Self-check of the library's bounded waits: one thread waits on an
// mbarrier that nothing arrives on, gives up after the wait bound
// (kWaitTimeoutNs, two seconds of global time), records kErrWaitTimeout in
// *status and returns, leaving the
// context usable. Nothing traps or faults.
__global__ void wait_probe_kernel(int* status) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t a = smem_u32(&bar);
  mbar_init(a, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  if (!mbar_wait(a, 0)) record_error(status, kErrWaitTimeout);
}

int wait_probe(int* status, cudaStream_t st) {
  if (status == nullptr) return set_error(TTRL_EINVAL, "wait_probe: null status");
  wait_probe_kernel<<<1, 1, 0, st>>>(status);
  note_launch();
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("wait_probe launch", e);
}

}  // namespace ttrl
