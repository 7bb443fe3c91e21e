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

// Each lane group of kLanes threads owns one (sequence, unit) pair of its CTA
// for the whole launch, so every index below is computed once. Within a step
// the group's lanes share the pair's side work: lane q stages one of the
// pair's inputs for the next step, stores to the peers q, q + kLanes, ..., and
// writes one of the pair's saved values to global memory.

// Shared-memory address of `local` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t peer_addr(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  return remote;
}

__device__ __forceinline__ void st_cluster(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Peers a lane stores to: q and q + kLanes (clusters have at most 16 CTAs).
constexpr int kPeersPerLane = 2;

__global__ void __launch_bounds__(1024) gru_seq_fwd_kernel(const __grid_constant__ GruSeqArgs a) {
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
  const int q = threadIdx.x & (kLanes - 1);
  const int p = threadIdx.x / kLanes;
  const bool active = p < rows * J;
  const int bl = active ? p / J : 0, jj = p - bl * J, j = j0 + jj, b = b0 + bl;
  const size_t plane = static_cast<size_t>(a.batch);
  // Lane q < 3 stages gi[s][b][q*H + j]; lane 3 of the unit-0 pair stages the
  // done flag entering step s + 1.
  auto stage = [&](int s, int buf) {
    if (!active) return;
    if (q < 3) {
      cp_async4(smem_u32(gs + (buf * R + bl) * 3 * J + q * J + jj),
                a.gi + (s * plane + b) * H3 + q * H + j, 4);
    } else if (q == 3 && jj == 0 && a.starts != nullptr && s + 1 < a.steps) {
      cp_async4(smem_u32(ss + buf * R + bl), a.starts + (s + 1) * plane + b, 4);
    }
  };
  stage(0, 0);
  cp_async_commit();
  cp_async_wait<0>();
  gru_cluster_sync();  // every CTA of the cluster is running before any peer store
  // This pair's element of each parity buffer in peers q and q + kLanes.
  const bool has0 = q < C, has1 = q + kLanes < C;
  const uint32_t ra0 = has0 ? peer_addr(hs + bl * ld + j, q) : 0u;
  const uint32_t rb0 = has0 ? peer_addr(hs + (R + bl) * ld + j, q) : 0u;
  const uint32_t ra1 = has1 ? peer_addr(hs + bl * ld + j, q + kLanes) : 0u;
  const uint32_t rb1 = has1 ? peer_addr(hs + (R + bl) * ld + j, q + kLanes) : 0u;
  const unsigned mask = group_mask();
  const int chunks = H >> 2;
  const float* wr = ws + jj * ld;
  const float* wz = ws + (J + jj) * ld;
  const float* wn = ws + (2 * J + jj) * ld;
  const float bhr = active ? a.b_hh[j] : 0.f;
  const float bhz = active ? a.b_hh[H + j] : 0.f;
  const float bhn = active ? a.b_hh[2 * H + j] : 0.f;
  for (int t = 0; t < a.steps; ++t) {
    const int cur = t & 1;
    const bool more = t + 1 < a.steps;
    if (more) stage(t + 1, cur ^ 1);
    cp_async_commit();
    float vq = 0.f;
    if (active) {
      const float* hrow = hs + (cur * R + bl) * ld;
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
      // Every lane of the group holds the sums and finishes the gates.
      const float* g3 = gs + (cur * R + bl) * 3 * J;
      const float ghr = __fadd_rn(ar, bhr);
      const float ghz = __fadd_rn(az, bhz);
      const float ghn = __fadd_rn(an, bhn);
      const float r = gru_sigmoid(__fadd_rn(g3[jj], ghr));
      const float z = gru_sigmoid(__fadd_rn(g3[J + jj], ghz));
      const float n = tanhf(__fadd_rn(g3[2 * J + jj], __fmul_rn(r, ghn)));
      const float hp = hrow[j];
      const float h = __fadd_rn(__fmul_rn(__fsub_rn(1.f, z), n), __fmul_rn(z, hp));
      const float hnext =
          (a.starts && more) ? __fmul_rn(h, __fsub_rn(1.f, ss[cur * R + bl])) : h;
      if (more) {
        if (has0) st_cluster(cur ? ra0 : rb0, hnext);
        if (has1) st_cluster(cur ? ra1 : rb1, hnext);
      }
      vq = q == 0 ? h : q == 1 ? hnext : q == 2 ? r : q == 3 ? z : q == 4 ? n
         : q == 5 ? ghr : q == 6 ? ghz : ghn;
    }
    // Publish the exchange and the staged inputs, then write this step's
    // saved activations while the barrier completes.
    cp_async_wait<0>();
    if (more) gru_cluster_arrive();
    if (active) {
      const size_t row = (t * plane + b) * H;
      const size_t row3 = (t * plane + b) * H3;
      if (q == 0) {
        a.out[row + j] = vq;
      } else if (q == 1) {
        if (more) a.hm[row + plane * H + j] = vq;
      } else if (q <= 4) {
        a.gates[row3 + (q - 2) * H + j] = vq;
      } else {
        a.gh[row3 + (q - 5) * H + j] = vq;
      }
    }
    if (more) gru_cluster_wait();
  }
}

__global__ void __launch_bounds__(1024) gru_seq_bwd_kernel(const __grid_constant__ GruSeqBwdArgs a) {
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
  float* xs = direct + R * J;        // [2][R][6J]: [dout | r | z | n | gh_n | hm] of a step
  float* ss = xs + 2 * R * 6 * J;    // [2][R]: done flag entering the step after
  for (int i = threadIdx.x; i < J * H3; i += blockDim.x) {
    const int jj = i / H3, c = i - jj * H3;
    wr[jj * ld + c] = a.w_hh[static_cast<size_t>(j0 + jj) * H3 + c];
  }
  const int q = threadIdx.x & (kLanes - 1);
  const int p = threadIdx.x / kLanes;
  const bool active = p < rows * J;
  const int bl = active ? p / J : 0, jj = p - bl * J, j = j0 + jj, b = b0 + bl;
  const size_t plane = static_cast<size_t>(a.batch);
  // Lane q < 6 stages field q of step s; lane 6 of the unit-0 pair stages the
  // done flag entering step s + 1.
  auto stage = [&](int s, int buf) {
    if (!active) return;
    const size_t r1 = s * plane + b;
    if (q < 6) {
      const float* src;
      uint32_t bytes = 4;
      if (q == 0) {
        src = a.dout ? a.dout + r1 * H + j : a.hm;  // no dout: zero-fill
        bytes = a.dout ? 4 : 0;
      } else if (q <= 3) {
        src = a.gates + r1 * H3 + (q - 1) * H + j;
      } else if (q == 4) {
        src = a.gh + r1 * H3 + 2 * H + j;
      } else {
        src = a.hm + r1 * H + j;
      }
      cp_async4(smem_u32(xs + (buf * R + bl) * 6 * J + q * J + jj), src, bytes);
    } else if (q == 6 && jj == 0 && a.starts != nullptr && s + 1 < a.steps) {
      cp_async4(smem_u32(ss + buf * R + bl), a.starts + (s + 1) * plane + b, 4);
    }
  };
  stage(a.steps - 1, 0);
  cp_async_commit();
  cp_async_wait<0>();
  gru_cluster_sync();
  const bool has0 = q < C, has1 = q + kLanes < C;
  const uint32_t ra0 = has0 ? peer_addr(ds + bl * ld + j, q) : 0u;
  const uint32_t rb0 = has0 ? peer_addr(ds + (R + bl) * ld + j, q) : 0u;
  const uint32_t ra1 = has1 ? peer_addr(ds + bl * ld + j, q + kLanes) : 0u;
  const uint32_t rb1 = has1 ? peer_addr(ds + (R + bl) * ld + j, q + kLanes) : 0u;
  const unsigned mask = group_mask();
  const int chunks = H3 >> 2;
  const float* wrow = wr + jj * ld;
  // Phases T-1 .. 0, then (when d h0 is wanted) a tail that reads step 0's d gh.
  const int phases = a.steps + (a.dh0 != nullptr ? 1 : 0);
  for (int it = 0; it < phases; ++it) {
    const bool tail = it == a.steps;
    const int t = tail ? 0 : a.steps - 1 - it;
    const int cur = it & 1;
    const bool carry = tail || t + 1 < a.steps;
    const bool push = it + 1 < phases;  // a later phase reads this step's d gh
    if (it + 1 < a.steps) stage(t - 1, cur ^ 1);
    cp_async_commit();
    float vq = 0.f;
    if (active) {
      float acc = 0.f;
      if (carry) {
        const float* drow = ds + (cur * R + bl) * ld;
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
          const float s0 = a.starts ? a.starts[b] : 0.f;
          a.dh0[static_cast<size_t>(b) * H + j] = a.starts ? dhm * (1.f - s0) : dhm;
        }
      } else {
        const float* x6 = xs + (cur * R + bl) * 6 * J;
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
          if (has0) {
            const uint32_t base = cur ? ra0 : rb0;
            st_cluster(base, dar);
            st_cluster(base + 4u * H, daz);
            st_cluster(base + 8u * H, dghn);
          }
          if (has1) {
            const uint32_t base = cur ? ra1 : rb1;
            st_cluster(base, dar);
            st_cluster(base + 4u * H, daz);
            st_cluster(base + 8u * H, dghn);
          }
        }
        if (q == 6) direct[bl * J + jj] = dh * z;
        // d gi = (d a_r, d a_z, d a_n); d gh = (d a_r, d a_z, d gh_n).
        vq = q == 0 ? dar : q == 1 ? daz : q == 2 ? dan : q == 3 ? dar : q == 4 ? daz : dghn;
      }
    }
    cp_async_wait<0>();
    if (push) gru_cluster_arrive();
    if (active && !tail && q < 6) {
      const size_t row3 = (t * plane + b) * H3;
      if (q < 3) a.dgi[row3 + q * H + j] = vq;
      else a.dgh[row3 + (q - 3) * H + j] = vq;
    }
    if (push) gru_cluster_wait();
  }
}

// Cluster size cap per device (16 where the hardware co-schedules it, else
// the portable 8), probed once by gru_init_device with both kernels' shared
// memory ceilings raised.
static int g_gru_cluster_cap[64];
constexpr size_t kGruSmemCap = 227u << 10;  // the per-CTA maximum on B200

struct GruSeqPlan {
  int csize, cols, rows, clusters, threads, ldh, ld3;
  size_t smem_fwd, smem_bwd;
};

// Row stride (floats) >= w with stride * 4 = 64 (mod 128) bytes, so the two
// lane groups of a quarter-warp reading adjacent rows hit disjoint banks.
static int gru_pad(int w) { return w + ((16 - w % 32) + 32) % 32; }

// The cluster size is the smallest of 4, 8, 16 whose per-CTA slices fit: a
// step's exchange costs more the more CTAs a cluster spans (measured on B200:
// about 0.56, 0.76 and 1.26 us per step at 4, 8 and 16 CTAs), while the
// per-lane work stays the same because the CTA's lane groups grow with it.
static bool gru_seq_plan(int batch, int hidden, GruSeqPlan* p) {
  if (batch <= 0 || hidden <= 0 || (hidden & 3) != 0) return false;
  int dev = 0;
  int cap = 8;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64 && g_gru_cluster_cap[dev] > 0)
    cap = g_gru_cluster_cap[dev];
  const int ldh = gru_pad(hidden), ld3 = gru_pad(3 * hidden);
  for (int c = 4; c <= cap && c <= kLanes * kPeersPerLane; c *= 2) {
    if (hidden % c != 0) continue;
    const int cols = hidden / c;
    const int most = 148 / c;
    const int rows = (batch + most - 1) / most;
    const int clusters = (batch + rows - 1) / rows;
    // One lane group per (sequence, unit) pair, a block of at most 1024 threads.
    const long long threads = ((static_cast<long long>(kLanes) * rows * cols + 31) / 32) * 32;
    if (threads > 1024) continue;
    const size_t rj = static_cast<size_t>(rows) * cols;
    const size_t fwd = ((static_cast<size_t>(3 * cols) + 2 * rows) * ldh + 2 * rj * 3 +
                        2 * rows) * sizeof(float);
    const size_t bwd = ((static_cast<size_t>(cols) + 2 * rows) * ld3 + rj + 2 * rj * 6 +
                        2 * rows) * sizeof(float);
    if (fwd > kGruSmemCap || bwd > kGruSmemCap) continue;
    *p = GruSeqPlan{c, cols, rows, clusters, static_cast<int>(threads), ldh, ld3, fwd, bwd};
    return true;
  }
  return false;
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
    cfg.blockDim = dim3(1024);
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
