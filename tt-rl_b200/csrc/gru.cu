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
// Those per-step kernels serve shapes the persistent sequence kernels below
// have no plan for; the sequence kernels run the whole unroll (and its
// backward) in one launch each.
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

// ------------------------------------------------- persistent sequence kernels
//
// The whole unroll in one launch, one thread-block cluster per slice of the
// sequences. The C CTAs of a cluster split the hidden units: CTA rank r owns
// J = H / C units j in [r * J, (r + 1) * J). The forward keeps the three gate
// columns of W_hh for its units in shared memory; the backward keeps the W_hh
// rows of its units. At every step a CTA computes its units for the cluster's
// sequences and pushes the result (the masked state entering the next step,
// or d gh of this step) straight into every peer's shared memory with
// st.shared::cluster; the cluster barrier (arrive.release / wait.acquire)
// publishes it. Nothing on the step-to-step path goes through global memory:
// the saved activations are written to global memory between the barrier's
// arrive and its wait, outside its release, so the barrier never waits for
// them. Sequences are independent, so clusters never wait on one another.
//
// Exchange buffers are double-buffered by step parity: a CTA writes the next
// step's buffer only after the barrier that ended every peer's reads of it.
// Each step's inputs that do not depend on the recurrence (gi forward; dout
// and the saved activations backward) are copied into shared memory one step
// ahead with cp.async, so their global latency hides behind the step before.
// Dot products run on the CUDA cores in fp32, kLanes threads per output, each
// over every kLanes-th float4 of the reduction, then a shuffle tree: a step
// is 2 x rows x 3H x H flops, far too small (M = rows) for the tensor cores,
// and the recurrence is bound by the latency of one exchange per step.

struct GruSeqArgs {
  const float* gi;      // [T][B][3H]
  const float* h0;      // [B][H]
  const float* starts;  // [T][B] or null
  const float* w_hh;    // [H][3H]
  const float* b_hh;    // [3H]
  float* gh;            // [T][B][3H]
  float* gates;         // [T][B][3H]
  float* hm;            // [T][B][H]
  float* out;           // [T][B][H]
  int steps, batch, hidden;
  int csize, cols, rows;  // CTAs per cluster, units per CTA, sequences per cluster
  int ldh, ld3;           // padded shared row strides for H and 3H
};

struct GruSeqBwdArgs {
  const float* dout;    // [T][B][H] or null
  const float* starts;  // [T][B] or null
  const float* w_hh;    // [H][3H]
  const float* gates;   // [T][B][3H]
  const float* gh;      // [T][B][3H]
  const float* hm;      // [T][B][H]
  float* dgi;           // [T][B][3H]
  float* dgh;           // [T][B][3H]
  float* dh0;           // [B][H] or null
  int steps, batch, hidden;
  int csize, cols, rows;
  int ldh, ld3;
};

__device__ __forceinline__ void gru_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The two halves of the cluster barrier: stores issued between them are not
// ordered by the release, so the barrier does not wait for them.
__device__ __forceinline__ void gru_cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void gru_cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t gru_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void st_peer(const float* local, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// Threads per output: each sums every kLanes-th float4 of the reduction,
// then a shuffle tree over the group.
constexpr int kLanes = 8;

__device__ __forceinline__ float group_sum(float v, unsigned mask) {
#pragma unroll
  for (int o = 1; o < kLanes; o <<= 1) v += __shfl_xor_sync(mask, v, o);
  return v;
}

__device__ __forceinline__ unsigned group_mask() {
  return ((1u << kLanes) - 1u) << (threadIdx.x & (32 - kLanes));
}

// The per-step inputs of the forward for this CTA's units and the cluster's
// rows, copied asynchronously: gi of step t ([R][3J]) and the done flag
// entering step t+1 ([R]).
__device__ __forceinline__ void fwd_stage(const GruSeqArgs& a, int t, float* gs, float* ss,
                                          int b0, int rows, int j0) {
  const int H = a.hidden, J = a.cols, H3 = 3 * H;
  for (int i = threadIdx.x; i < rows * 3 * J; i += blockDim.x) {
    const int bl = i / (3 * J), cl = i - bl * 3 * J;
    const float* src = a.gi + (static_cast<size_t>(t) * a.batch + b0 + bl) * H3 + (cl / J) * H +
                       j0 + (cl % J);
    cp_async4(smem_u32(gs + i), src, 4);
  }
  if (a.starts != nullptr && t + 1 < a.steps) {
    for (int i = threadIdx.x; i < rows; i += blockDim.x)
      cp_async4(smem_u32(ss + i), a.starts + static_cast<size_t>(t + 1) * a.batch + b0 + i, 4);
  }
  cp_async_commit();
}

__global__ void __launch_bounds__(512) gru_seq_fwd_kernel(const __grid_constant__ GruSeqArgs a) {
  extern __shared__ __align__(16) float smem[];
  pdl_trigger();
  pdl_wait();
  const int H = a.hidden, J = a.cols, H3 = 3 * H, ld = a.ldh, R = a.rows, C = a.csize;
  const int rank = static_cast<int>(gru_cluster_rank());
  const int j0 = rank * J;
  const int b0 = (blockIdx.x / C) * R;
  const int rows = min(R, a.batch - b0);
  float* ws = smem;                // [3J][ld]: column g*H + j0 + jj of W_hh
  float* hs = ws + 3 * J * ld;     // [2][R][ld]: the state entering a step, by parity
  float* gs = hs + 2 * R * ld;     // [2][R][3J]: gi of a step, by parity
  float* ss = gs + 2 * R * 3 * J;  // [2][R]: done flag entering the next step
  float* res = ss + 2 * R;         // [2][8][R][J]: h, hm next, r, z, n, gh r z n, by parity
  // W_hh row k holds this CTA's J columns of each gate contiguously: read
  // them unit-fastest (coalesced) and transpose into ws.
  for (int i = threadIdx.x; i < 3 * J * H; i += blockDim.x) {
    const int k = i / (3 * J), cl = i - k * 3 * J, g = cl / J, jj = cl - g * J;
    ws[cl * ld + k] = a.w_hh[static_cast<size_t>(k) * H3 + g * H + j0 + jj];
  }
  for (int i = threadIdx.x; i < rows * H; i += blockDim.x) {
    const int bl = i / H, k = i - bl * H, b = b0 + bl;
    const float h = a.h0[static_cast<size_t>(b) * H + k];
    const float v = a.starts ? __fmul_rn(h, __fsub_rn(1.f, a.starts[b])) : h;
    hs[bl * ld + k] = v;
    if (k >= j0 && k < j0 + J) a.hm[static_cast<size_t>(b) * H + k] = v;
  }
  fwd_stage(a, 0, gs, ss, b0, rows, j0);
  cp_async_wait<0>();
  gru_cluster_sync();  // every CTA of the cluster is running before any peer store
  const int q = threadIdx.x & (kLanes - 1);
  const unsigned mask = group_mask();
  const int chunks = H >> 2;
  const size_t plane = static_cast<size_t>(a.batch);
  for (int t = 0; t < a.steps; ++t) {
    const int cur = t & 1;
    const float* hc = hs + cur * R * ld;
    float* hn = hs + (cur ^ 1) * R * ld;
    const float* gc = gs + cur * R * 3 * J;
    float* rc = res + cur * 8 * R * J;
    const bool more = t + 1 < a.steps;
    if (more) fwd_stage(a, t + 1, gs + (cur ^ 1) * R * 3 * J, ss + (cur ^ 1) * R, b0, rows, j0);
    for (int p = threadIdx.x / kLanes; p < rows * J; p += blockDim.x / kLanes) {
      const int bl = p / J, jj = p - bl * J, j = j0 + jj;
      const float* hrow = hc + bl * ld;
      const float* wr = ws + jj * ld;
      const float* wz = ws + (J + jj) * ld;
      const float* wn = ws + (2 * J + jj) * ld;
      float ar = 0.f, az = 0.f, an = 0.f;
      for (int c = q; c < chunks; c += kLanes) {
        const float4 h4 = *reinterpret_cast<const float4*>(hrow + 4 * c);
        const float4 r4 = *reinterpret_cast<const float4*>(wr + 4 * c);
        const float4 z4 = *reinterpret_cast<const float4*>(wz + 4 * c);
        const float4 n4 = *reinterpret_cast<const float4*>(wn + 4 * c);
        ar = fmaf(h4.x, r4.x, ar); ar = fmaf(h4.y, r4.y, ar);
        ar = fmaf(h4.z, r4.z, ar); ar = fmaf(h4.w, r4.w, ar);
        az = fmaf(h4.x, z4.x, az); az = fmaf(h4.y, z4.y, az);
        az = fmaf(h4.z, z4.z, az); az = fmaf(h4.w, z4.w, az);
        an = fmaf(h4.x, n4.x, an); an = fmaf(h4.y, n4.y, an);
        an = fmaf(h4.z, n4.z, an); an = fmaf(h4.w, n4.w, an);
      }
      ar = group_sum(ar, mask);
      az = group_sum(az, mask);
      an = group_sum(an, mask);
      // Every lane of the group holds the sums; each finishes the gates and
      // takes a share of the stores.
      const float* g3 = gc + bl * 3 * J;
      const float ghr = __fadd_rn(ar, a.b_hh[j]);
      const float ghz = __fadd_rn(az, a.b_hh[H + j]);
      const float ghn = __fadd_rn(an, a.b_hh[2 * H + j]);
      const float r = gru_sigmoid(__fadd_rn(g3[jj], ghr));
      const float z = gru_sigmoid(__fadd_rn(g3[J + jj], ghz));
      const float n = tanhf(__fadd_rn(g3[2 * J + jj], __fmul_rn(r, ghn)));
      const float hp = hrow[j];
      const float h = __fadd_rn(__fmul_rn(__fsub_rn(1.f, z), n), __fmul_rn(z, hp));
      const float hnext =
          (a.starts && more) ? __fmul_rn(h, __fsub_rn(1.f, ss[cur * R + bl])) : h;
      if (more) {
        for (int peer = q; peer < C; peer += kLanes) st_peer(hn + bl * ld + j, peer, hnext);
      }
      float vq;
      switch (q) {
        case 0: vq = h; break;
        case 1: vq = hnext; break;
        case 2: vq = r; break;
        case 3: vq = z; break;
        case 4: vq = n; break;
        case 5: vq = ghr; break;
        case 6: vq = ghz; break;
        default: vq = ghn; break;
      }
      rc[(q * R + bl) * J + jj] = vq;
    }
    // Publish the exchange (and the staged next-step inputs), then write the
    // step's saved activations while the barrier completes.
    cp_async_wait<0>();
    __syncthreads();
    if (more) gru_cluster_arrive();
    for (int i = threadIdx.x; i < 8 * rows * J; i += blockDim.x) {
      const int f = i / (rows * J), rem = i - f * rows * J, bl = rem / J, jj = rem - bl * J;
      const int b = b0 + bl, j = j0 + jj;
      const float v = rc[(f * R + bl) * J + jj];
      const size_t row = (t * plane + b) * H;
      const size_t row3 = (t * plane + b) * H3;
      if (f == 0) {
        a.out[row + j] = v;
      } else if (f == 1) {
        if (more) a.hm[row + plane * H + j] = v;
      } else if (f <= 4) {
        a.gates[row3 + (f - 2) * H + j] = v;
      } else {
        a.gh[row3 + (f - 5) * H + j] = v;
      }
    }
    if (more) gru_cluster_wait();
  }
}

// The per-step inputs of the backward for this CTA's units and the cluster's
// rows: per row [dout | r | z | n | gh_n | hm] (J each) and the done flag
// entering step t+1.
__device__ __forceinline__ void bwd_stage(const GruSeqBwdArgs& a, int t, float* xs, float* ss,
                                          int b0, int rows, int j0) {
  const int H = a.hidden, J = a.cols, H3 = 3 * H;
  for (int i = threadIdx.x; i < rows * 6 * J; i += blockDim.x) {
    const int bl = i / (6 * J), cl = i - bl * 6 * J, f = cl / J, jj = cl - f * J;
    const size_t r1 = static_cast<size_t>(t) * a.batch + b0 + bl;
    const float* src;
    uint32_t bytes = 4;
    if (f == 0) {
      src = a.dout ? a.dout + r1 * H + j0 + jj : a.hm;  // no dout: zero-fill
      bytes = a.dout ? 4 : 0;
    } else if (f <= 3) {
      src = a.gates + r1 * H3 + (f - 1) * H + j0 + jj;
    } else if (f == 4) {
      src = a.gh + r1 * H3 + 2 * H + j0 + jj;
    } else {
      src = a.hm + r1 * H + j0 + jj;
    }
    cp_async4(smem_u32(xs + i), src, bytes);
  }
  if (a.starts != nullptr && t + 1 < a.steps) {
    for (int i = threadIdx.x; i < rows; i += blockDim.x)
      cp_async4(smem_u32(ss + i), a.starts + static_cast<size_t>(t + 1) * a.batch + b0 + i, 4);
  }
  cp_async_commit();
}

__global__ void __launch_bounds__(512) gru_seq_bwd_kernel(const __grid_constant__ GruSeqBwdArgs a) {
  extern __shared__ __align__(16) float smem[];
  pdl_trigger();
  pdl_wait();
  const int H = a.hidden, J = a.cols, H3 = 3 * H, ld = a.ld3, R = a.rows, C = a.csize;
  const int rank = static_cast<int>(gru_cluster_rank());
  const int j0 = rank * J;
  const int b0 = (blockIdx.x / C) * R;
  const int rows = min(R, a.batch - b0);
  float* wr = smem;                  // [J][ld]: row j0 + jj of W_hh
  float* ds = wr + J * ld;           // [2][R][ld]: d gh of the step after, by parity
  float* direct = ds + 2 * R * ld;   // [R][J]: dh * z of the step after
  float* xs = direct + R * J;        // [2][R][6J]: staged per-step inputs
  float* ss = xs + 2 * R * 6 * J;    // [2][R]: done flag entering the step after
  float* res = ss + 2 * R;           // [2][4][R][J]: d a_r, d a_z, d a_n, d gh_n, by parity
  for (int i = threadIdx.x; i < J * H3; i += blockDim.x) {
    const int jj = i / H3, c = i - jj * H3;
    wr[jj * ld + c] = a.w_hh[static_cast<size_t>(j0 + jj) * H3 + c];
  }
  bwd_stage(a, a.steps - 1, xs, ss, b0, rows, j0);
  cp_async_wait<0>();
  gru_cluster_sync();
  const int q = threadIdx.x & (kLanes - 1);
  const unsigned mask = group_mask();
  const int chunks = H3 >> 2;
  const size_t plane = static_cast<size_t>(a.batch);
  // Phases T-1 .. 0, then (when d h0 is wanted) a tail that reads step 0's d gh.
  const int phases = a.steps + (a.dh0 != nullptr ? 1 : 0);
  for (int it = 0; it < phases; ++it) {
    const bool tail = it == a.steps;
    const int t = tail ? 0 : a.steps - 1 - it;
    const int cur = it & 1;
    const bool carry = tail || t + 1 < a.steps;
    const bool push = it + 1 < phases;  // a later phase reads this step's d gh
    const float* dc = ds + cur * R * ld;
    float* dn_buf = ds + (cur ^ 1) * R * ld;
    const float* xc = xs + cur * R * 6 * J;
    float* rc = res + cur * 4 * R * J;
    if (it + 1 < a.steps)
      bwd_stage(a, t - 1, xs + (cur ^ 1) * R * 6 * J, ss + (cur ^ 1) * R, b0, rows, j0);
    for (int p = threadIdx.x / kLanes; p < rows * J; p += blockDim.x / kLanes) {
      const int bl = p / J, jj = p - bl * J, j = j0 + jj;
      float acc = 0.f;
      if (carry) {
        const float* drow = dc + bl * ld;
        const float* wrow = wr + jj * ld;
        for (int c = q; c < chunks; c += kLanes) {
          const float4 d4 = *reinterpret_cast<const float4*>(drow + 4 * c);
          const float4 w4 = *reinterpret_cast<const float4*>(wrow + 4 * c);
          acc = fmaf(d4.x, w4.x, acc); acc = fmaf(d4.y, w4.y, acc);
          acc = fmaf(d4.z, w4.z, acc); acc = fmaf(d4.w, w4.w, acc);
        }
        acc = group_sum(acc, mask);
      }
      const float dhm = carry ? direct[bl * J + jj] + acc : 0.f;
      if (tail) {
        if (q == 0) {
          const int b = b0 + bl;
          const float s0 = a.starts ? a.starts[b] : 0.f;
          a.dh0[static_cast<size_t>(b) * H + j] = a.starts ? dhm * (1.f - s0) : dhm;
        }
        continue;
      }
      const float* x6 = xc + bl * 6 * J;
      float dh = x6[jj];
      if (carry) dh += a.starts ? dhm * (1.f - ss[cur * R + bl]) : dhm;
      const float r = x6[J + jj], z = x6[2 * J + jj], n = x6[3 * J + jj];
      const float ghn = x6[4 * J + jj], hp = x6[5 * J + jj];
      const float dnn = dh * (1.f - z);
      const float dz = dh * (hp - n);
      const float dan = dnn * (1.f - n * n);
      const float dar = (dan * ghn) * r * (1.f - r);
      const float daz = dz * z * (1.f - z);
      const float dghn = dan * r;
      if (push) {
        float* dst = dn_buf + bl * ld;
        for (int peer = q; peer < C; peer += kLanes) {
          st_peer(dst + j, peer, dar);
          st_peer(dst + H + j, peer, daz);
          st_peer(dst + 2 * H + j, peer, dghn);
        }
      }
      if (q < 4) {
        const float vq = q == 0 ? dar : (q == 1 ? daz : (q == 2 ? dan : dghn));
        rc[(q * R + bl) * J + jj] = vq;
      } else if (q == 4) {
        direct[bl * J + jj] = dh * z;
      }
    }
    cp_async_wait<0>();
    __syncthreads();
    if (push) gru_cluster_arrive();
    if (!tail) {
      // d gi = (d a_r, d a_z, d a_n); d gh = (d a_r, d a_z, d gh_n).
      for (int i = threadIdx.x; i < 6 * rows * J; i += blockDim.x) {
        const int f = i / (rows * J), rem = i - f * rows * J, bl = rem / J, jj = rem - bl * J;
        const int b = b0 + bl, j = j0 + jj;
        const size_t row3 = (t * plane + b) * H3;
        if (f < 3) {
          a.dgi[row3 + f * H + j] = rc[(f * R + bl) * J + jj];
        } else {
          const int g = f - 3;
          a.dgh[row3 + g * H + j] = rc[((g == 2 ? 3 : g) * R + bl) * J + jj];
        }
      }
    }
    if (push) gru_cluster_wait();
  }
}

// Cluster size cap per device (16 where the hardware co-schedules it, else
// the portable 8), probed once by gru_init_device with both kernels' shared
// memory ceilings raised.
static int g_gru_cluster_cap[64];
constexpr size_t kGruSmemCap = 200u << 10;

struct GruSeqPlan {
  int csize, cols, rows, clusters, threads, ldh, ld3;
  size_t smem_fwd, smem_bwd;
};

// Row stride (floats) >= w with stride * 4 = 64 (mod 128) bytes, so the two
// lane groups of a quarter-warp reading adjacent rows hit disjoint banks.
static int gru_pad(int w) { return w + ((16 - w % 32) + 32) % 32; }

static bool gru_seq_plan(int batch, int hidden, GruSeqPlan* p) {
  if (batch <= 0 || hidden <= 0 || (hidden & 3) != 0) return false;
  int dev = 0;
  int cap = 8;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64 && g_gru_cluster_cap[dev] > 0)
    cap = g_gru_cluster_cap[dev];
  int c = cap;
  while (c > 1 && hidden % c != 0) c >>= 1;
  const int cols = hidden / c;
  int most = 148 / c;
  if (most < 1) most = 1;
  const int rows = (batch + most - 1) / most;
  const int clusters = (batch + rows - 1) / rows;
  long long threads = ((static_cast<long long>(kLanes) * rows * cols + 31) / 32) * 32;
  if (threads > 512) threads = 512;
  const int ldh = gru_pad(hidden), ld3 = gru_pad(3 * hidden);
  const size_t rj = static_cast<size_t>(rows) * cols;
  const size_t fwd = ((static_cast<size_t>(3 * cols) + 2 * rows) * ldh + 2 * rj * 3 + 2 * rows +
                      2 * 8 * rj) * sizeof(float);
  const size_t bwd = ((static_cast<size_t>(cols) + 2 * rows) * ld3 + rj + 2 * rj * 6 + 2 * rows +
                      2 * 4 * rj) * sizeof(float);
  if (fwd > kGruSmemCap || bwd > kGruSmemCap) return false;
  *p = GruSeqPlan{c, cols, rows, clusters, static_cast<int>(threads), ldh, ld3, fwd, bwd};
  return true;
}

int gru_init_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
  const int most = static_cast<int>(kGruSmemCap);
  e = cudaFuncSetAttribute(gru_seq_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gru_seq_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
  if (e != cudaSuccess) return set_cuda_error("gru attributes", e);
  int cap = 8;
  if (cudaFuncSetAttribute(gru_seq_fwd_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
          cudaSuccess &&
      cudaFuncSetAttribute(gru_seq_bwd_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
          cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(16);
    cfg.blockDim = dim3(512);
    cfg.dynamicSmemBytes = kGruSmemCap;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 16;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int fits_fwd = 0, fits_bwd = 0;
    if (cudaOccupancyMaxActiveClusters(&fits_fwd, gru_seq_fwd_kernel, &cfg) == cudaSuccess &&
        cudaOccupancyMaxActiveClusters(&fits_bwd, gru_seq_bwd_kernel, &cfg) == cudaSuccess &&
        fits_fwd >= 1 && fits_bwd >= 1)
      cap = 16;
  }
  cudaGetLastError();  // a refused probe leaves no sticky error
  if (dev >= 0 && dev < 64) g_gru_cluster_cap[dev] = cap;
  return TTRL_OK;
}

template <typename Args>
static cudaError_t launch_clustered(void (*kernel)(Args), const GruSeqPlan& p, size_t smem,
                                    cudaStream_t st, const Args& args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.clusters * p.csize);
  cfg.blockDim = dim3(p.threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, args);
}

int gru_seq_fwd(const GruSeqArgs& in, cudaStream_t st) {
  GruSeqPlan p;
  if (in.steps <= 0) return set_error(TTRL_EINVAL, "gru_sequence_fwd: steps must be > 0");
  if (!gru_seq_plan(in.batch, in.hidden, &p))
    return set_error(TTRL_EUNSUPPORTED, "gru_sequence_fwd: batch %d x hidden %d has no plan",
                     in.batch, in.hidden);
  if (!in.gi || !in.h0 || !in.w_hh || !in.b_hh || !in.gh || !in.gates || !in.hm || !in.out)
    return set_error(TTRL_EINVAL, "gru_sequence_fwd: null pointer");
  GruSeqArgs a = in;
  a.csize = p.csize;
  a.cols = p.cols;
  a.rows = p.rows;
  a.ldh = p.ldh;
  a.ld3 = p.ld3;
  cudaError_t e = launch_clustered(gru_seq_fwd_kernel, p, p.smem_fwd, st, a);
  note_launch();
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("gru_sequence_fwd launch", e);
}

int gru_seq_bwd(const GruSeqBwdArgs& in, cudaStream_t st) {
  GruSeqPlan p;
  if (in.steps <= 0) return set_error(TTRL_EINVAL, "gru_sequence_bwd: steps must be > 0");
  if (!gru_seq_plan(in.batch, in.hidden, &p))
    return set_error(TTRL_EUNSUPPORTED, "gru_sequence_bwd: batch %d x hidden %d has no plan",
                     in.batch, in.hidden);
  if (!in.w_hh || !in.gates || !in.gh || !in.hm || !in.dgi || !in.dgh)
    return set_error(TTRL_EINVAL, "gru_sequence_bwd: null pointer");
  GruSeqBwdArgs a = in;
  a.csize = p.csize;
  a.cols = p.cols;
  a.rows = p.rows;
  a.ldh = p.ldh;
  a.ld3 = p.ld3;
  cudaError_t e = launch_clustered(gru_seq_bwd_kernel, p, p.smem_bwd, st, a);
  note_launch();
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("gru_sequence_bwd launch", e);
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

int ttrl_gru_sequence_supported(int batch, int hidden) {
  GruSeqPlan p;
  return gru_seq_plan(batch, hidden, &p) ? 1 : 0;
}

int ttrl_gru_sequence_fwd(const float* gi, const float* h0, const float* starts,
                          const float* w_hh, const float* b_hh, float* gh, float* gates, float* hm,
                          float* out, int steps, int batch, int hidden, ttrl_stream_t stream) {
  GruSeqArgs a{gi, h0, starts, w_hh, b_hh, gh, gates, hm, out, steps, batch, hidden,
               0, 0, 0, 0, 0};
  return gru_seq_fwd(a, static_cast<cudaStream_t>(stream));
}

int ttrl_gru_sequence_bwd(const float* dout, const float* starts, const float* w_hh,
                          const float* gates, const float* gh, const float* hm, float* dgi,
                          float* dgh, float* dh0, int steps, int batch, int hidden,
                          ttrl_stream_t stream) {
  GruSeqBwdArgs a{dout, starts, w_hh, gates, gh, hm, dgi, dgh, dh0, steps, batch, hidden,
                  0, 0, 0, 0, 0};
  return gru_seq_bwd(a, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
