// tcgen05 GEMM for the learner update: D[r][c] = sum_k A[r][k] * B[c][k].
//
// One CTA owns a 128 x BN tile of D held in TMEM and walks its share of K
// in 32-wide k-blocks through a ring of shared-memory stages: eight loader
// warps gather each stage with cp.async (and, for split-TF32, split the
// chunks they copied), then arrive on the stage's "full" mbarrier; a ninth
// warp waits on it and issues the tcgen05.mma instructions, whose commit
// frees the stage again. No block-wide barrier sits in the main loop. Each operand is *gathered* (dense strided matrix, convolution
// im2col, or transposed im2col for the weight gradient), so one kernel
// serves Linear fwd/dgrad/wgrad and Conv2d fprop/dgrad/wgrad without
// materialising any im2col buffer. Tiles land in the canonical swizzled
// layouts (K-major SWIZZLE_128B, or MN-major SWIZZLE_128B_BASE32B for 32-bit
// operands) depending on which dimension is contiguous in global memory,
// and thread 0 issues tcgen05.mma.kind::tf32.
//
// Gather addressing is split into a per-CTA part (each thread's rows or row
// chunk, computed once) and a per-k-block part (multiply-shift division, no
// hardware divides), which keeps the load path a few instructions per
// 16-byte copy.
//
// Precision: TTRL_PREC_TF32X3 splits every operand into a tf32 high part and
// an fp32 remainder in shared memory and accumulates hi*hi + hi*lo + lo*hi,
// which reproduces fp32 products to ~1e-6 relative. TTRL_PREC_TF32 issues a
// single pass on the truncated operands.
//
// K can be split across CTAs (blockIdx.z). Each split writes its partial
// tile to the workspace; the last CTA of a tile to arrive (a device counter,
// left at zero afterwards) sums the partials in split order and applies the
// epilogue, so results are deterministic and no second kernel is launched.
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

constexpr int kLoadWarps = 8;
constexpr int kThreads = 256;                       // loader threads
constexpr int kBlockThreads = kThreads + 32;        // + the MMA warp
constexpr int kMmaWarp = kLoadWarps;

// Constant sources for the synthetic "ones" row an operand may append: a
// GEMM whose A operand carries a row of ones produces the column sums of B
// (the bias gradient) in that row of D.
__device__ __align__(16) float kOnes4[4] = {1.f, 1.f, 1.f, 1.f};
__device__ __align__(16) float kOneZeros[4] = {1.f, 0.f, 0.f, 0.f};

__device__ __forceinline__ int fdiv(const FastDiv& f, int n) {
  if (f.shr == 0) return n;  // divisor 1
  const uint32_t t = __umulhi(static_cast<uint32_t>(n), f.mul);
  return static_cast<int>((t + static_cast<uint32_t>(n)) >> f.shr);
}

// General element address (used by the scalar fallback modes only).
__device__ const float* opnd_addr(const DevOperand& o, int r, int k, bool& ok) {
  ok = false;
  if (k >= o.kdim) return o.ptr;
  if (r >= o.rows) {
    if (o.ones_row && r == o.rows) {
      ok = true;
      return kOnes4;
    }
    return o.ptr;
  }
  if (o.kind == TTRL_OPND_DENSE) {
    ok = true;
    return o.ptr + static_cast<long long>(r) * o.rs + static_cast<long long>(k) * o.ks;
  }
  const int m = o.kind == TTRL_OPND_CONV_FPROP ? r : k;
  const int q = o.kind == TTRL_OPND_CONV_FPROP ? k : r;
  const int img = fdiv(o.f_ohw, m);
  const int rem = m - img * o.oh * o.ow;
  const int oy = fdiv(o.f_ow, rem);
  const int ox = rem - oy * o.ow;
  const int t = fdiv(o.f_c, q);
  const int c = q - t * o.c;
  const int ky = fdiv(o.f_kw, t);
  const int kx = t - ky * o.kw;
  const int iy = oy * o.stride - o.pad + ky;
  const int ix = ox * o.stride - o.pad + kx;
  if (iy < 0 || iy >= o.h || ix < 0 || ix >= o.w) return o.ptr;
  ok = true;
  return o.ptr + ((static_cast<long long>(img) * o.h + iy) * o.w + ix) * o.c + c;
}

// Per-thread gather state for one operand tile of R rows. In the vector
// modes each thread owns R/32 copies per k-block: K-major (kModeKVec) keeps
// a fixed 4-wide k chunk and R/32 rows; MN-major (kModeMNVec) keeps a fixed
// 4-row chunk and R/32 k lines.
template <int R>
struct Loader {
  static constexpr int P = R / 32;
  static constexpr int RC = R / 4;
  long long off[P];  // KVec: element offset of each row's (window) origin
  int iy0[P], ix0[P];
  uint32_t valid, ones;
  long long coff;  // MNVec: offset of the thread's row chunk
  int cky, ckx;
  bool cvalid, cones;

  __device__ void init(const DevOperand& o, int row0, int tid) {
    valid = ones = 0;
    coff = 0;
    cky = ckx = 0;
    cvalid = cones = false;
    if (o.mode == kModeKVec) {
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const int r = row0 + (tid >> 3) + i * 32;
        off[i] = 0;
        iy0[i] = ix0[i] = 0;
        if (r < o.rows) {
          valid |= 1u << i;
          if (o.kind == TTRL_OPND_DENSE) {
            off[i] = static_cast<long long>(r) * o.rs;
          } else {
            const int img = fdiv(o.f_ohw, r);
            const int rem = r - img * o.oh * o.ow;
            const int oy = fdiv(o.f_ow, rem);
            const int ox = rem - oy * o.ow;
            iy0[i] = oy * o.stride - o.pad;
            ix0[i] = ox * o.stride - o.pad;
            off[i] = ((static_cast<long long>(img) * o.h + iy0[i]) * o.w + ix0[i]) * o.c;
          }
        } else if (o.ones_row && r == o.rows) {
          ones |= 1u << i;
        }
      }
    } else if (o.mode == kModeMNVec) {
      const int r = row0 + (tid % RC) * 4;
      cvalid = r < o.rows;
      cones = !cvalid && o.ones_row && r == o.rows;
      if (cvalid) {
        if (o.kind == TTRL_OPND_DENSE) {
          coff = r;  // rs == 1 in this mode
        } else {
          const int t = fdiv(o.f_c, r);
          const int c = r - t * o.c;
          cky = fdiv(o.f_kw, t);
          ckx = t - cky * o.kw;
          coff = c;
        }
      }
    }
  }

  __device__ void issue(const DevOperand& o, uint32_t base, int row0, int k0, int tid) {
    if (o.mode == kModeKVec) {
      const int kc = tid & 7;
      const int k = k0 + kc * 4;
      const bool kvalid = k < o.kdim;
      long long koff = k;
      int ky = 0, kx = 0;
      if (o.kind != TTRL_OPND_DENSE) {
        const int t = fdiv(o.f_c, k);
        const int c = k - t * o.c;
        ky = fdiv(o.f_kw, t);
        kx = t - ky * o.kw;
        koff = (static_cast<long long>(ky) * o.w + kx) * o.c + c;
      }
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const int rl = (tid >> 3) + i * 32;
        bool ok = kvalid && ((valid >> i) & 1u);
        if (ok && o.kind != TTRL_OPND_DENSE) {
          const int iy = iy0[i] + ky, ix = ix0[i] + kx;
          ok = iy >= 0 && iy < o.h && ix >= 0 && ix < o.w;
        }
        const bool one = kvalid && ((ones >> i) & 1u);
        const float* src = ok ? o.ptr + off[i] + koff : (one ? kOnes4 : o.ptr);
        cp_async16(base + kmajor_off(rl, kc * 4), src, (ok || one) ? 16u : 0u);
      }
    } else if (o.mode == kModeMNVec) {
      const int rc = tid % RC;
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const int k = tid / RC + i * (kThreads / RC);
        const int kg = k0 + k;
        bool ok = cvalid && kg < o.kdim;
        const float* src = o.ptr;
        if (ok) {
          if (o.kind == TTRL_OPND_DENSE) {
            src = o.ptr + coff + static_cast<long long>(kg) * o.ks;
          } else {
            const int img = fdiv(o.f_ohw, kg);
            const int rem = kg - img * o.oh * o.ow;
            const int oy = fdiv(o.f_ow, rem);
            const int ox = rem - oy * o.ow;
            const int iy = oy * o.stride - o.pad + cky;
            const int ix = ox * o.stride - o.pad + ckx;
            ok = iy >= 0 && iy < o.h && ix >= 0 && ix < o.w;
            src = ok ? o.ptr + ((static_cast<long long>(img) * o.h + iy) * o.w + ix) * o.c + coff
                     : o.ptr;
          }
        }
        const bool one = cones && kg < o.kdim;
        if (one) src = kOneZeros;
        cp_async16(base + mnmajor_off(rc * 4, k), src, (ok || one) ? 16u : 0u);
      }
    } else {
      // Scalar fallback (odd extents or alignment): 4-byte gathers into a
      // K-major tile.
      const bool rows_fast = o.mode == kModeScalarR;
#pragma unroll 4
      for (int t = tid; t < R * 32; t += kThreads) {
        const int r = rows_fast ? t % R : t >> 5;
        const int k = rows_fast ? t / R : t & 31;
        bool ok;
        const float* src = opnd_addr(o, row0 + r, k0 + k, ok);
        cp_async4(base + kmajor_off(r, k), src, ok ? 4u : 0u);
      }
    }
  }

  // Split the chunks this thread copied for one stage: hi (tf32-exact) in
  // place in the raw tile, lo = x - hi at the same offset in the low tile.
  __device__ void split(const DevOperand& o, uint8_t* hi_gen, uint8_t* lo_gen, int tid) const {
    if (o.mode == kModeKVec || o.mode == kModeMNVec) {
      uint32_t off[P];
      float4 x[P];
#pragma unroll
      for (int i = 0; i < P; ++i) {
        off[i] = o.mode == kModeKVec
                     ? kmajor_off((tid >> 3) + i * 32, (tid & 7) * 4)
                     : mnmajor_off((tid % RC) * 4, tid / RC + i * (kThreads / RC));
        x[i] = *reinterpret_cast<const float4*>(hi_gen + off[i]);
      }
#pragma unroll
      for (int i = 0; i < P; ++i) {
        float4 hi, lo;
        split_tf32(x[i].x, hi.x, lo.x);
        split_tf32(x[i].y, hi.y, lo.y);
        split_tf32(x[i].z, hi.z, lo.z);
        split_tf32(x[i].w, hi.w, lo.w);
        *reinterpret_cast<float4*>(hi_gen + off[i]) = hi;
        *reinterpret_cast<float4*>(lo_gen + off[i]) = lo;
      }
    } else {
      const bool rows_fast = o.mode == kModeScalarR;
      for (int t = tid; t < R * 32; t += kThreads) {
        const int r = rows_fast ? t % R : t >> 5;
        const int k = rows_fast ? t / R : t & 31;
        const uint32_t off = kmajor_off(r, k);
        float hi, lo;
        split_tf32(*reinterpret_cast<const float*>(hi_gen + off), hi, lo);
        *reinterpret_cast<float*>(hi_gen + off) = hi;
        *reinterpret_cast<float*>(lo_gen + off) = lo;
      }
    }
  }
};

__device__ __forceinline__ void epi_store(const ttrl_epilogue& ep, const EpiExtra& ex, int r,
                                          int c, float acc) {
  if (ex.row2 >= 0 && r == ex.row2) {
    // The synthetic ones row: column sums of B, stored unscaled.
    float* o = ex.out2 + static_cast<long long>(c) * ex.cs2;
    float v = acc;
    if (ex.accumulate2) v += *o;
    *o = v;
    return;
  }
  float v = ep.alpha * acc;
  if (ep.bias_mode == TTRL_BIAS_ROW) {
    v += ep.bias[r];
  } else if (ep.bias_mode == TTRL_BIAS_COL) {
    v += ep.bias[c];
  }
  if (ep.mask != nullptr) {
    if (!(ep.mask[static_cast<long long>(r) * ep.mrs + static_cast<long long>(c) * ep.mcs] > 0.f))
      v = 0.f;
  }
  if (ep.relu) v = v > 0.f ? v : 0.f;
  float* o = ep.out + static_cast<long long>(r) * ep.ors + static_cast<long long>(c) * ep.ocs;
  if (ep.accumulate) v += *o;
  *o = v;
}

template <int BN, bool SPLIT>
struct TileCfg {
  static constexpr int kABytes = 128 * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kTile = kABytes + kBBytes;  // one raw (or lo) stage
  // Split-TF32 keeps the low parts in a short ring of their own, so the
  // raw ring can be deep: more k-blocks in flight per CTA.
  static constexpr int kLoSlots = SPLIT ? (BN >= 128 ? 2 : 3) : 0;
  static constexpr int kBudget = 196 * 1024 - kLoSlots * kTile;
  static constexpr int kRawFit = kBudget / kTile;
  static constexpr int kStages = kRawFit > 8 ? 8 : kRawFit;
  // A raw stage is refilled once the MMAs of the k-block two iterations
  // back have drained, so the tensor pipe's latency stays off the load path.
  static constexpr int kLag = kStages >= 4 ? 2 : 1;
  static constexpr int kAhead = kStages - kLag;  // k-blocks in flight
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem =
      (kStages + kLoSlots) * kTile + 1024 /*align slack*/ + 512 /*barriers*/;
  static_assert(kStages >= 3, "at least three pipeline stages");
  static_assert(kStages * kTile >= 128 * (BN + 1) * 4, "epilogue staging fits in the ring");
};

// Named barrier over the 256 loader threads (the MMA warp does not join).
__device__ __forceinline__ void loader_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
}

template <int BN, bool SPLIT>
__global__ void __launch_bounds__(kBlockThreads, 1)
    gemm_tc_kernel(const __grid_constant__ GemmArgs args) {
  using Cfg = TileCfg<BN, SPLIT>;
  constexpr int S = Cfg::kStages;
  constexpr int L = Cfg::kLoSlots;
  constexpr int LL = L > 0 ? L : 1;  // divisor-safe in the non-split build
  constexpr int AHEAD = Cfg::kAhead;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_last;
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t sbase = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_u32);
  const uint32_t lo_base = sbase + S * Cfg::kTile;
  const uint32_t empty0 = lo_base + L * Cfg::kTile;  // S "raw stage free"
  const uint32_t full0 = empty0 + S * 8;              // S "stage ready for MMA"
  const uint32_t loempty0 = full0 + S * 8;            // L "lo slot free"
  const uint32_t accum_bar = loempty0 + (L > 0 ? L : 1) * 8;
  const uint32_t tmem_slot = accum_bar + 8;
  const uint32_t* tmem_slot_gen =
      reinterpret_cast<const uint32_t*>(sgen + (tmem_slot - sbase));

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(empty0 + s * 8, 1);
      mbar_init(full0 + s * 8, kLoadWarps);
    }
    for (int l = 0; l < L; ++l) mbar_init(loempty0 + l * 8, 1);
    mbar_init(accum_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }

  const int row0 = blockIdx.x * 128;
  const int col0 = blockIdx.y * BN;
  const int kb0 = blockIdx.z * args.kb_per_split;
  const int kb1 = min(args.kblocks, kb0 + args.kb_per_split);
  const int nk = kb1 - kb0;
  const bool a_mn = args.a.mode == kModeMNVec;
  const bool b_mn = args.b.mode == kModeMNVec;
  const bool split_a = SPLIT && !args.a.exact;
  const bool split_b = SPLIT && !args.b.exact;
  bool timed_out = false;

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_gen;

  auto raw_a = [&](int s) { return sbase + s * Cfg::kTile; };
  auto raw_b = [&](int s) { return sbase + s * Cfg::kTile + Cfg::kABytes; };

  if (warp < kLoadWarps) {
    // ---- loader warps ----
    Loader<128> la;
    Loader<BN> lb;
    la.init(args.a, row0, tid);
    lb.init(args.b, col0, tid);
#pragma unroll 1
    for (int s = 0; s < AHEAD; ++s) {
      if (s < nk) {
        la.issue(args.a, raw_a(s), row0, (kb0 + s) * 32, tid);
        lb.issue(args.b, raw_b(s), col0, (kb0 + s) * 32, tid);
      }
      cp_async_commit();
    }
#pragma unroll 1
    for (int i = 0; i < nk; ++i) {
      const int j = i + AHEAD;
      if (j < nk) {
        const int sj = j % S;
        if (j >= S) {
          // Raw stage sj was last read by the MMAs of k-block j - S.
          if (!mbar_wait(empty0 + sj * 8, ((j - S) / S) & 1)) timed_out = true;
        }
        la.issue(args.a, raw_a(sj), row0, (kb0 + j) * 32, tid);
        lb.issue(args.b, raw_b(sj), col0, (kb0 + j) * 32, tid);
      }
      cp_async_commit();
      cp_async_wait<AHEAD>();  // this thread's copies of k-block i have landed
      const int s = i % S;
      if (split_a || split_b) {
        const int l = i % LL;
        if (i >= L) {
          // Lo slot l was last read by the MMAs of k-block i - L.
          if (!mbar_wait(loempty0 + l * 8, ((i - L) / LL) & 1)) timed_out = true;
        }
        uint8_t* hi = sgen + s * Cfg::kTile;
        uint8_t* lo = sgen + (lo_base - sbase) + l * Cfg::kTile;
        if (split_a) la.split(args.a, hi, lo, tid);
        if (split_b) lb.split(args.b, hi + Cfg::kABytes, lo + Cfg::kABytes, tid);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(full0 + s * 8);
    }
  } else if (lane == 0) {
    // ---- MMA warp: one thread issues every tcgen05.mma of the tile ----
    const uint32_t idesc = idesc_tf32(128, BN, a_mn, b_mn);
    const uint32_t albo = a_mn ? 4096u : 16u, blbo = b_mn ? 4096u : 16u;
    const uint32_t asbo = a_mn ? 512u : 1024u, bsbo = b_mn ? 512u : 1024u;
    const uint32_t alay = a_mn ? kLayoutSw128Base32 : kLayoutSw128;
    const uint32_t blay = b_mn ? kLayoutSw128Base32 : kLayoutSw128;
    // Descriptors of raw stage 0 / lo slot 0; stage, slot and k-step
    // offsets only move the start-address field (addresses stay below
    // 256 KB, so no carry leaves it).
    const uint64_t da = umma_desc(raw_a(0), albo, asbo, alay);
    const uint64_t db = umma_desc(raw_b(0), blbo, bsbo, blay);
    const uint64_t lo_off = (lo_base - sbase) >> 4;
    const uint64_t astep = a_mn ? 1024 >> 4 : 32 >> 4;
    const uint64_t bstep = b_mn ? 1024 >> 4 : 32 >> 4;
#pragma unroll 1
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      const int l = i % LL;
      if (!mbar_wait(full0 + s * 8, (i / S) & 1)) timed_out = true;
      tc_fence_after();
      const uint64_t so = static_cast<uint64_t>(s) * (Cfg::kTile >> 4);
      const uint64_t lso = lo_off + static_cast<uint64_t>(l) * (Cfg::kTile >> 4);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t ad = da + so + ks * astep;
        const uint64_t bd = db + so + ks * bstep;
        umma_tf32(tmem, ad, bd, idesc, (i > 0 || ks > 0) ? 1u : 0u);
        if (split_b) umma_tf32(tmem, ad, bd - so + lso, idesc, 1u);
        if (split_a) umma_tf32(tmem, ad - so + lso, bd, idesc, 1u);
      }
      umma_commit(empty0 + s * 8);
      if (L > 0) umma_commit(loempty0 + l * 8);
    }
    umma_commit(accum_bar);
  }

  // ---- epilogue: TMEM -> registers -> staged tile in shared memory ->
  // coalesced stores (the pipeline ring is idle once the accumulator is
  // ready, so the tile reuses it) ----
  const bool split_k = args.ws != nullptr;
  const int rows = min(128, args.m - row0);
  const int cols = min(BN, args.n - col0);
  constexpr int LD = BN + 1;  // padded row: conflict-free in both passes
  float* tile = reinterpret_cast<float*>(sgen);
  if (warp < kLoadWarps) {
    if (!mbar_wait(accum_bar, 0)) timed_out = true;
    tc_fence_after();
    {
      const int rl = (warp & 3) * 32 + lane;
      const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
      const int cbeg = (warp >> 2) * (BN / 2);
#pragma unroll 1
      for (int c = cbeg; c < cbeg + BN / 2; c += 8) {
        if (c >= cols) break;  // uniform across the warp
        float v[8];
        tmem_ld8(trow + c, v);
#pragma unroll
        for (int q = 0; q < 8; ++q) tile[rl * LD + c + q] = v[q];
      }
    }
    loader_sync();
    if (timed_out) {
      record_error(args.status, kErrWaitTimeout);
    } else if (split_k) {
      float* wz = args.ws + static_cast<long long>(blockIdx.z) * args.m * args.n;
      for (int e = tid; e < rows * cols; e += kThreads) {
        const int rl = e / cols, c = e - rl * cols;
        wz[static_cast<long long>(row0 + rl) * args.n + col0 + c] = tile[rl * LD + c];
      }
    } else if (args.ep.ocs == 1 || args.ep.ors != 1) {
      for (int e = tid; e < rows * cols; e += kThreads) {
        const int rl = e / cols, c = e - rl * cols;
        epi_store(args.ep, args.ex, row0 + rl, col0 + c, tile[rl * LD + c]);
      }
    } else {
      // Transposed output (ors == 1): walk rows fastest.
      for (int e = tid; e < rows * cols; e += kThreads) {
        const int c = e / rows, rl = e - c * rows;
        epi_store(args.ep, args.ex, row0 + rl, col0 + c, tile[rl * LD + c]);
      }
    }
  } else if (timed_out) {
    record_error(args.status, kErrWaitTimeout);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, Cfg::kTmemCols);

  if (split_k && args.reduce_in_kernel) {
    // The last split CTA of this tile sums every partial in split order.
    const int tile_id = blockIdx.y * gridDim.x + blockIdx.x;
    if (tid == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(reinterpret_cast<unsigned*>(args.counters) + tile_id, 1u);
      s_last = (prev == gridDim.z - 1) ? 1 : 0;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      const long long plane = static_cast<long long>(args.m) * args.n;
      for (int e = tid; e < rows * cols; e += kBlockThreads) {
        const int rr = row0 + e / cols, cc = col0 + e % cols;
        const float* p = args.ws + static_cast<long long>(rr) * args.n + cc;
        float sum = 0.f;
        for (unsigned z = 0; z < gridDim.z; ++z) sum += __ldcg(p + z * plane);
        epi_store(args.ep, args.ex, rr, cc, sum);
      }
      if (tid == 0) args.counters[tile_id] = 0;
    }
  }
}

// Sum split-K partials in split order and apply the epilogue (used when the
// partial tiles are too large for one CTA to reduce quickly).
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int m, int n,
                                     ttrl_epilogue ep, EpiExtra ex) {
  const long long total = static_cast<long long>(m) * n;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(idx / n);
    const int c = static_cast<int>(idx - static_cast<long long>(r) * n);
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += ws[static_cast<long long>(sp) * total + idx];
    epi_store(ep, ex, r, c, s);
  }
}

// ------------------------------------------------------------------ host

template <int BN, bool SPLIT>
static int set_smem_attr() {
  using Cfg = TileCfg<BN, SPLIT>;
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, SPLIT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("cudaFuncSetAttribute(gemm)", e);
}

int gemm_init_device() {
  int rc = TTRL_OK;
  if ((rc = set_smem_attr<32, true>())) return rc;
  if ((rc = set_smem_attr<64, true>())) return rc;
  if ((rc = set_smem_attr<128, true>())) return rc;
  if ((rc = set_smem_attr<32, false>())) return rc;
  if ((rc = set_smem_attr<64, false>())) return rc;
  if ((rc = set_smem_attr<128, false>())) return rc;
  return TTRL_OK;
}

FastDiv make_fastdiv(int d) {
  FastDiv f;
  f.d = static_cast<uint32_t>(d < 1 ? 1 : d);
  if (f.d == 1) {
    f.mul = 0;
    f.shr = 0;
    return f;
  }
  uint32_t l = 0;
  while ((1ull << l) < f.d) ++l;
  f.mul = static_cast<uint32_t>(((1ull << 32) * ((1ull << l) - f.d)) / f.d + 1);
  f.shr = l;
  return f;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Pick the gather mode of an operand from its strides and alignment.
static int resolve_operand(const ttrl_operand& in, int ones_row, DevOperand& out) {
  std::memset(&out, 0, sizeof(out));
  out.ptr = static_cast<const float*>(in.ptr);
  out.kind = in.kind;
  out.rows = in.rows;
  out.kdim = in.kdim;
  out.rs = in.rs;
  out.ks = in.ks;
  out.n = in.n;
  out.h = in.h;
  out.w = in.w;
  out.c = in.c;
  out.kh = in.kh;
  out.kw = in.kw;
  out.stride = in.stride;
  out.pad = in.pad;
  out.oh = in.oh;
  out.ow = in.ow;
  out.ones_row = ones_row;
  out.exact = (in.flags & TTRL_OPND_EXACT_TF32) ? 1 : 0;
  if (in.ptr == nullptr && in.rows > 0 && in.kdim > 0)
    return set_error(TTRL_EINVAL, "gemm operand has a null pointer");
  if (in.kind == TTRL_OPND_DENSE) {
    const bool al = aligned16(in.ptr);
    if (in.ks == 1 && in.kdim % 4 == 0 && in.rs % 4 == 0 && al) {
      out.mode = kModeKVec;
    } else if (in.rs == 1 && in.rows % 4 == 0 && in.ks % 4 == 0 && al) {
      out.mode = kModeMNVec;
    } else {
      out.mode = (in.rs <= in.ks && in.rs != 0) ? kModeScalarR : kModeScalarK;
    }
    return TTRL_OK;
  }
  if (in.kind == TTRL_OPND_CONV_FPROP || in.kind == TTRL_OPND_CONV_WGRAD) {
    if (in.n <= 0 || in.h <= 0 || in.w <= 0 || in.c <= 0 || in.kh <= 0 || in.kw <= 0 ||
        in.stride <= 0 || in.pad < 0 || in.oh <= 0 || in.ow <= 0)
      return set_error(TTRL_EINVAL, "gemm conv operand has an invalid geometry");
    const long long span = static_cast<long long>(in.n) * in.h * in.w * in.c;
    if (span >= (1ll << 31) || static_cast<long long>(in.n) * in.oh * in.ow >= (1ll << 31))
      return set_error(TTRL_EUNSUPPORTED, "gemm conv operand exceeds 2^31 elements");
    out.f_ohw = make_fastdiv(in.oh * in.ow);
    out.f_ow = make_fastdiv(in.ow);
    out.f_c = make_fastdiv(in.c);
    out.f_kw = make_fastdiv(in.kw);
    const bool vec = (in.c % 4 == 0) && aligned16(in.ptr);
    if (in.kind == TTRL_OPND_CONV_FPROP)
      out.mode = vec ? kModeKVec : kModeScalarK;
    else
      out.mode = vec ? kModeMNVec : kModeScalarR;
    return TTRL_OK;
  }
  return set_error(TTRL_EINVAL, "gemm operand kind %d is unknown", in.kind);
}

static int pick_bn(int n) {
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  return 128;
}

struct Schedule {
  int bn, kblocks, splits, kb_per_split, tiles;
};

static Schedule make_schedule(const ttrl_gemm_desc& d) {
  Schedule s;
  s.bn = pick_bn(d.n);
  s.kblocks = (d.k + 31) / 32;
  s.tiles = ((d.m + 127) / 128) * ((d.n + s.bn - 1) / s.bn);
  int splits = d.splits;
  if (splits <= 0) {
    // Aim for about one wave of 148 SMs, at least 4 k-blocks per CTA, and
    // at most 32 partials for the last CTA of a tile to reduce.
    splits = 1;
    if (s.tiles < 120 && s.kblocks >= 8) {
      const int want = (148 + s.tiles - 1) / s.tiles;
      const int most = s.kblocks / 4;
      splits = want < most ? want : most;
      if (splits > 32) splits = 32;
      if (splits < 1) splits = 1;
    }
  }
  if (splits > s.kblocks) splits = s.kblocks > 0 ? s.kblocks : 1;
  s.kb_per_split = (s.kblocks + splits - 1) / splits;
  if (s.kb_per_split < 1) s.kb_per_split = 1;
  s.splits = (s.kblocks + s.kb_per_split - 1) / s.kb_per_split;
  if (s.splits < 1) s.splits = 1;
  return s;
}

size_t gemm_workspace_bytes(const ttrl_gemm_desc& d) {
  const Schedule s = make_schedule(d);
  if (s.splits <= 1) return kCounterBytes;
  return kCounterBytes + static_cast<size_t>(s.splits) * d.m * d.n * sizeof(float);
}

template <int BN, bool SPLIT>
static cudaError_t launch_bn(const GemmArgs& args, dim3 grid, cudaStream_t stream) {
  using Cfg = TileCfg<BN, SPLIT>;
  gemm_tc_kernel<BN, SPLIT><<<grid, kBlockThreads, Cfg::kSmem, stream>>>(args);
  note_launch();
  return cudaGetLastError();
}

int gemm_run(const ttrl_gemm_desc& d, int a_ones_row, const EpiExtra& ex, int* counters,
             float* partials, size_t partial_bytes, int* status, cudaStream_t stream) {
  if (d.m < 0 || d.n < 0 || d.k < 0) return set_error(TTRL_EINVAL, "gemm: negative extent");
  if (d.m == 0 || d.n == 0) return TTRL_OK;
  if (d.ep.out == nullptr) return set_error(TTRL_EINVAL, "gemm: null output");
  if (d.precision != TTRL_PREC_TF32X3 && d.precision != TTRL_PREC_TF32)
    return set_error(TTRL_EINVAL, "gemm: unknown precision %d", d.precision);
  if (d.k == 0) return set_error(TTRL_EUNSUPPORTED, "gemm: empty reduction (k == 0)");

  GemmArgs args;
  std::memset(&args, 0, sizeof(args));
  int rc;
  if ((rc = resolve_operand(d.a, a_ones_row, args.a))) return rc;
  if ((rc = resolve_operand(d.b, 0, args.b))) return rc;
  if (args.a.rows + (a_ones_row ? 1 : 0) < d.m || args.b.rows < d.n)
    return set_error(TTRL_EINVAL, "gemm: operand rows smaller than the output extent");
  args.ep = d.ep;
  args.ex = ex;
  args.m = d.m;
  args.n = d.n;
  args.k = d.k;
  args.status = status;

  const Schedule s = make_schedule(d);
  args.kblocks = s.kblocks;
  args.kb_per_split = s.kb_per_split;
  if (s.splits > 1) {
    const size_t need = static_cast<size_t>(s.splits) * d.m * d.n * sizeof(float);
    if (counters == nullptr || partials == nullptr || partial_bytes < need)
      return set_error(TTRL_EWORKSPACE, "gemm: needs %zu bytes of workspace, got %zu",
                       need + kCounterBytes, partial_bytes + kCounterBytes);
    if (s.tiles > static_cast<int>(kCounterBytes / sizeof(int)))
      return set_error(TTRL_EUNSUPPORTED, "gemm: %d split tiles exceed the counter space",
                       s.tiles);
    args.counters = counters;
    args.ws = partials;
    // One CTA sums at most ~32K partial values in the kernel's tail; larger
    // reductions go to a parallel second kernel.
    args.reduce_in_kernel = static_cast<long long>(s.splits) * s.bn * 128 <= 32 * 1024;
  }
  dim3 grid((d.m + 127) / 128, (d.n + s.bn - 1) / s.bn, s.splits);
  const bool split3 = d.precision == TTRL_PREC_TF32X3;
  cudaError_t e;
  switch (s.bn) {
    case 32: e = split3 ? launch_bn<32, true>(args, grid, stream) : launch_bn<32, false>(args, grid, stream); break;
    case 64: e = split3 ? launch_bn<64, true>(args, grid, stream) : launch_bn<64, false>(args, grid, stream); break;
    default: e = split3 ? launch_bn<128, true>(args, grid, stream) : launch_bn<128, false>(args, grid, stream); break;
  }
  if (e != cudaSuccess) return set_cuda_error("gemm launch", e);
  if (s.splits > 1 && !args.reduce_in_kernel) {
    const long long total = static_cast<long long>(d.m) * d.n;
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > 148 * 8) blocks = 148 * 8;
    splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(args.ws, s.splits, d.m, d.n, d.ep, ex);
    note_launch();
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gemm split-k reduce launch", e);
  }
  return TTRL_OK;
}

}  // namespace ttrl
