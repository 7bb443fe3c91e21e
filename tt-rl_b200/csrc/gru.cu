// The GRU unroll's per-step pointwise work, fused (ttrl/engine/recurrent.py:86-94
// and :143-168). A step of the unroll is
//   gh_t = hm_t @ W_hh + b_hh                       (tcgen05 GEMM, gemm_tc.cu)
//   r = sigmoid(gi_r + gh_r); z = sigmoid(gi_z + gh_z)
//   n = tanh(gi_n + r * gh_n); h_t = (1 - z) * n + z * hm_t
//   hm_{t+1} = h_t * (1 - start_{t+1})              (the done mask entering t+1)
// where gi = x @ W_ih + b_ih for every timestep comes from one GEMM over the
// whole sequence before the loop. gru_fwd_kernel is everything after the GEMM
// in one launch, with each operation rounded as the reference's op-by-op
// composition rounds it (no contraction into fma), so the fused step gives
// the same bits as the composed ops on the same gi, gh.
//
// The backward walks t = T-1 .. 0. gru_bwd_kernel takes d h_t (the heads'
// gradient plus the carry from step t+1 through that step's done mask),
// produces d gi_t and d gh_t, and leaves dh * z (the direct path into hm_t)
// in the carry buffer, onto which the caller accumulates d gh_t @ W_hh^T
// with one GEMM. The weight gradients of both GEMMs then come from one
// GEMM each over all T steps.
//
// Gate columns follow PyTorch's order: [reset | update | candidate], each
// `hidden` wide, rows [batch][3 * hidden].
#include "common.cuh"
#include "internal.h"

namespace ttrl {

struct GruFwdArgs {
  const float* gi;
  const float* gh;
  const float* hm;
  const float* start_next;
  float* out;
  float* gates;
  float* hm_next;
  int batch;
  int hidden;
};

struct GruBwdArgs {
  const float* dout;
  float* dhm;
  const float* start_next;
  const float* gates;
  const float* gh;
  const float* hm;
  float* dgi;
  float* dgh;
  int batch;
  int hidden;
  int carry;
};

__device__ __forceinline__ float gru_sigmoid(float x) { return 1.f / (1.f + expf(-x)); }

__global__ void gru_fwd_kernel(const __grid_constant__ GruFwdArgs a) {
  pdl_trigger();
  pdl_wait();
  const int h3 = 3 * a.hidden;
  const int total = a.batch * a.hidden;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int b = i / a.hidden, j = i - b * a.hidden;
    const float* gi = a.gi + static_cast<size_t>(b) * h3;
    const float* gh = a.gh + static_cast<size_t>(b) * h3;
    const float r = gru_sigmoid(__fadd_rn(gi[j], gh[j]));
    const float z = gru_sigmoid(__fadd_rn(gi[a.hidden + j], gh[a.hidden + j]));
    const float n = tanhf(__fadd_rn(gi[2 * a.hidden + j], __fmul_rn(r, gh[2 * a.hidden + j])));
    const float hp = a.hm[i];
    const float h = __fadd_rn(__fmul_rn(__fsub_rn(1.f, z), n), __fmul_rn(z, hp));
    a.out[i] = h;
    float* g = a.gates + static_cast<size_t>(b) * h3;
    g[j] = r;
    g[a.hidden + j] = z;
    g[2 * a.hidden + j] = n;
    if (a.hm_next != nullptr)
      a.hm_next[i] = a.start_next ? __fmul_rn(h, __fsub_rn(1.f, a.start_next[b])) : h;
  }
}

__global__ void gru_bwd_kernel(const __grid_constant__ GruBwdArgs a) {
  pdl_trigger();
  pdl_wait();
  const int h3 = 3 * a.hidden;
  const int total = a.batch * a.hidden;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int b = i / a.hidden, j = i - b * a.hidden;
    float dh = a.dout ? a.dout[i] : 0.f;
    if (a.carry) {
      const float c = a.dhm[i];
      dh += a.start_next ? c * (1.f - a.start_next[b]) : c;
    }
    const float* g = a.gates + static_cast<size_t>(b) * h3;
    const float r = g[j], z = g[a.hidden + j], n = g[2 * a.hidden + j];
    const float ghn = a.gh[static_cast<size_t>(b) * h3 + 2 * a.hidden + j];
    const float hp = a.hm[i];
    // h = (1 - z) n + z hp
    const float dn = dh * (1.f - z);
    const float dz = dh * (hp - n);
    // n = tanh(gi_n + r gh_n); r, z = sigmoid(.)
    const float dan = dn * (1.f - n * n);
    const float dar = (dan * ghn) * r * (1.f - r);
    const float daz = dz * z * (1.f - z);
    float* dgi = a.dgi + static_cast<size_t>(b) * h3;
    float* dgh = a.dgh + static_cast<size_t>(b) * h3;
    dgi[j] = dar;
    dgi[a.hidden + j] = daz;
    dgi[2 * a.hidden + j] = dan;
    dgh[j] = dar;
    dgh[a.hidden + j] = daz;
    dgh[2 * a.hidden + j] = dan * r;
    a.dhm[i] = dh * z;
  }
}

__global__ void gru_mask_kernel(const float* __restrict__ h, const float* __restrict__ start,
                                float* __restrict__ out, int batch, int hidden) {
  pdl_trigger();
  pdl_wait();
  const int total = batch * hidden;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int b = i / hidden;
    out[i] = start ? __fmul_rn(h[i], __fsub_rn(1.f, start[b])) : h[i];
  }
}

static int gru_blocks(int batch, int hidden) {
  const long long total = static_cast<long long>(batch) * hidden;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

static int gru_check(int batch, int hidden, const char* what) {
  if (batch <= 0 || hidden <= 0)
    return set_error(TTRL_EINVAL, "%s: batch %d and hidden %d must be > 0", what, batch, hidden);
  if (static_cast<long long>(batch) * 3 * hidden > (1LL << 30))
    return set_error(TTRL_EINVAL, "%s: batch x 3 x hidden exceeds 2^30", what);
  return TTRL_OK;
}

int gru_fwd(const GruFwdArgs& a, cudaStream_t st) {
  int rc = gru_check(a.batch, a.hidden, "gru_gates_fwd");
  if (rc != TTRL_OK) return rc;
  if (!a.gi || !a.gh || !a.hm || !a.out || !a.gates)
    return set_error(TTRL_EINVAL, "gru_gates_fwd: null pointer");
  const cudaError_t le = launch_pdl(gru_fwd_kernel, dim3(gru_blocks(a.batch, a.hidden)), dim3(256),
                                    0, st, a);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("gru_gates_fwd launch", e);
}

int gru_bwd(const GruBwdArgs& a, cudaStream_t st) {
  int rc = gru_check(a.batch, a.hidden, "gru_gates_bwd");
  if (rc != TTRL_OK) return rc;
  if (!a.dhm || !a.gates || !a.gh || !a.hm || !a.dgi || !a.dgh)
    return set_error(TTRL_EINVAL, "gru_gates_bwd: null pointer");
  const cudaError_t le = launch_pdl(gru_bwd_kernel, dim3(gru_blocks(a.batch, a.hidden)), dim3(256),
                                    0, st, a);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("gru_gates_bwd launch", e);
}

int gru_mask(const float* h, const float* start, float* out, int batch, int hidden,
             cudaStream_t st) {
  int rc = gru_check(batch, hidden, "gru_mask");
  if (rc != TTRL_OK) return rc;
  if (!h || !out) return set_error(TTRL_EINVAL, "gru_mask: null pointer");
  const cudaError_t le = launch_pdl(gru_mask_kernel, dim3(gru_blocks(batch, hidden)), dim3(256),
                                    0, st, h, start, out, batch, hidden);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("gru_mask launch", e);
}

}  // namespace ttrl

using namespace ttrl;

extern "C" {

int ttrl_gru_gates_fwd(const float* gi, const float* gh, const float* hm, const float* start_next,
                       float* out, float* gates, float* hm_next, int batch, int hidden,
                       ttrl_stream_t stream) {
  GruFwdArgs a{gi, gh, hm, start_next, out, gates, hm_next, batch, hidden};
  return gru_fwd(a, static_cast<cudaStream_t>(stream));
}

int ttrl_gru_gates_bwd(const float* dout, float* dhm, const float* start_next, int carry,
                       const float* gates, const float* gh, const float* hm, float* dgi,
                       float* dgh, int batch, int hidden, ttrl_stream_t stream) {
  GruBwdArgs a{dout, dhm, start_next, gates, gh, hm, dgi, dgh, batch, hidden, carry};
  return gru_bwd(a, static_cast<cudaStream_t>(stream));
}

int ttrl_gru_mask(const float* h, const float* start, float* out, int batch, int hidden,
                  ttrl_stream_t stream) {
  return gru_mask(h, start, out, batch, hidden, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
