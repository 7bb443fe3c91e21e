// tcgen05 GEMM for the learner update: D[r][c] = sum_k A[r][k] * B[c][k].
//
// One CTA owns a 128 x BN tile of D held in TMEM and walks its share of K
// in 32-wide k-blocks through a ring of shared-memory stages. Warp roles:
//   - a TMA producer warp (one elected lane) loads every operand that is a
//     plain dense matrix with 16-byte-aligned strides with
//     cp.async.bulk.tensor, refilling a stage as soon as the MMA frees it;
//   - eight loader warps *gather* the other operands with cp.async: the
//     convolution im2col, the transposed im2col of the weight gradient, and
//     dense matrices TMA cannot describe. So one kernel serves Linear
//     fwd/dgrad/wgrad and Conv2d fprop/dgrad/wgrad without materialising any
//     im2col buffer. For split-TF32 the loader warps also write each stage's
//     low part into a separate ring;
//   - one MMA warp (one elected lane) issues tcgen05.mma.kind::tf32 and
//     commits each stage back to its "empty" mbarrier.
// No block-wide barrier sits in the main loop. Tiles land in the canonical
// swizzled layouts (K-major SWIZZLE_128B, or MN-major SWIZZLE_128B_BASE32B
// for 32-bit operands) depending on which dimension is contiguous in global
// memory; TMA writes the same layouts.
//
// Gather addressing is split into a per-CTA part (each thread's rows or row
// chunk, computed once) and a per-k-block part (multiply-shift division, no
// hardware divides), which keeps the load path a few instructions per
// 16-byte copy.
//
// Precision: TTRL_PREC_TF32X3 accumulates hi*hi + hi*lo + lo*hi. The MMA
// reads fp32 operands and uses their tf32 part, so the raw stage is the high
// part and only lo = x - tf32(x) is written; this reproduces fp32 products
// to ~1e-6 relative. TTRL_PREC_TF32 issues a single pass over operands the
// loader warps first round to the nearest tf32 in shared memory (the MMA's
// own truncation is biased and its error would accumulate along K).
//
// Split-K (blockIdx.z): up to 16 splits run as one thread-block cluster and
// reduce their partial tiles through distributed shared memory in split
// order. Very long K (>= 32 k-blocks per split at the cluster limit) splits
// up to 64 ways through a global workspace instead; the last CTA of a tile to
// arrive (a device counter, left at zero afterwards) sums the partials in
// split order, or splitk_reduce_kernel does when the partials are large.
// Either way results are deterministic. Grids of several waves use a
// half-footprint variant (SMALL) that fits two CTAs per SM.
//
// Every launch uses programmatic dependent launch: TMEM allocation and
// barrier set-up overlap the previous kernel's tail, and griddepcontrol.wait
// precedes the first global access.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

constexpr int kLoadWarps = 8;
constexpr int kThreads = 256;                       // loader threads
constexpr int kBlockThreads = kThreads + 64;        // + the MMA warp + the TMA producer warp
constexpr int kMmaWarp = kLoadWarps;
constexpr int kProducerWarp = kLoadWarps + 1;
// When both operands arrive by TMA, the loader warps form this many groups
// that take alternate k-blocks, each covering a whole stage, so that several
// stages' split or rounding passes are in flight at once. A pass is bound by
// shared-memory load latency (the loads queue behind the tensor core's own
// operand reads), not by its bytes, so one stage at a time would serialise
// that latency into every k-block.
constexpr int kLoaderGroups = 2;
constexpr int kGroupWarps = kLoadWarps / kLoaderGroups;
constexpr int kGroupThreads = kGroupWarps * 32;

// Largest cluster (in split CTAs) the split-K reduction may use on each
// device: 16 where the hardware can co-schedule it, else the portable 8.
// Written by gemm_init_device.
static int g_max_cluster[64];

// How many clusters of each size (2..16 split CTAs) of the full-footprint
// variant can be resident at once on each device, per tile width (32, 64,
// 128) and precision (single pass, split-TF32); 0 where not queried.
// Written by gemm_init_device.
static int g_active_clusters[64][3][2][17];

// Constant sources for the synthetic "ones" row an operand may append: a
// GEMM whose A operand carries a row of ones produces the column sums of B
// (the bias gradient) in that row of D.
__device__ __align__(16) float kOnes4[4] = {1.f, 1.f, 1.f, 1.f};
__device__ __align__(16) float kOneZeros[4] = {1.f, 0.f, 0.f, 0.f};


// 16-byte shared-memory load and store on a 32-bit shared-window address.
// The loader warps address stages this way: a generic pointer into shared
// memory costs an address-space resolution on every access.
__device__ __forceinline__ float4 lds4(uint32_t saddr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(saddr)
               : "memory");
  return v;
}
__device__ __forceinline__ void sts4(uint32_t saddr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(saddr), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

// General element address (used by the scalar fallback modes only).
__device__ __forceinline__ const float* opnd_addr(const DevOperand& o, int r, int k, bool& ok) {
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

  __device__ __forceinline__ void init(const DevOperand& o, int row0, int tid) {
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

  __device__ __forceinline__ void issue(const DevOperand& o, uint32_t base, int row0, int k0,
                                        int tid) {
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

  // The synthetic ones row of an MN-major operand whose stage arrived by TMA
  // (which cannot produce it): 1.0 at every valid k of tile row
  // `o.rows - row0`, 0.0 past the end of K. Written by the threads that split
  // those chunks, before they read them.
  __device__ __forceinline__ void fill_ones_row(const DevOperand& o, uint8_t* raw_gen, int row0,
                                                int k0, int tid) const {
    const int r = o.rows - row0;
    if (r < 0 || r >= R || (tid % RC) != (r >> 2)) return;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int k = tid / RC + i * (kThreads / RC);
      *reinterpret_cast<float*>(raw_gen + mnmajor_off(r, k)) = k0 + k < o.kdim ? 1.f : 0.f;
    }
  }

  // Single-pass precision: round the chunks this thread owns (the ones
  // `split` would read) to tf32 in place.
  __device__ __forceinline__ void round_in_place(const DevOperand& o, uint8_t* raw_gen,
                                                 uint32_t raw_s, int tid) const {
    if (o.mode == kModeKVec || o.mode == kModeMNVec) {
      uint32_t off[P];
      float4 x[P];
#pragma unroll
      for (int i = 0; i < P; ++i) {
        off[i] = raw_s + (o.mode == kModeKVec
                              ? kmajor_off((tid >> 3) + i * 32, (tid & 7) * 4)
                              : mnmajor_off((tid % RC) * 4, tid / RC + i * (kThreads / RC)));
        x[i] = lds4(off[i]);
      }
#pragma unroll
      for (int i = 0; i < P; ++i) {
        x[i].x = tf32_round(x[i].x);
        x[i].y = tf32_round(x[i].y);
        x[i].z = tf32_round(x[i].z);
        x[i].w = tf32_round(x[i].w);
        sts4(off[i], x[i]);
      }
    } else {
      const bool rows_fast = o.mode == kModeScalarR;
      for (int t = tid; t < R * 32; t += kThreads) {
        const int r = rows_fast ? t % R : t >> 5;
        const int k = rows_fast ? t / R : t & 31;
        float* p = reinterpret_cast<float*>(raw_gen + kmajor_off(r, k));
        *p = tf32_round(*p);
      }
    }
  }

  // Split the chunks this thread copied for one stage. tcgen05.mma of kind
  // tf32 reads an fp32 operand as its high 19 bits (the low 13 bits are
  // ignored, i.e. truncated), so the raw stage already is the high part;
  // only the remainder lo = x - trunc(x) is written, to the low tile at the
  // same offset.
  __device__ __forceinline__ void split(const DevOperand& o, const uint8_t* raw_gen,
                                        uint8_t* lo_gen, uint32_t raw_s, uint32_t lo_s,
                                        int tid) const {
    if (o.mode == kModeKVec || o.mode == kModeMNVec) {
      uint32_t off[P];
      float4 x[P];
#pragma unroll
      for (int i = 0; i < P; ++i) {
        off[i] = o.mode == kModeKVec
                     ? kmajor_off((tid >> 3) + i * 32, (tid & 7) * 4)
                     : mnmajor_off((tid % RC) * 4, tid / RC + i * (kThreads / RC));
        x[i] = lds4(raw_s + off[i]);
      }
#pragma unroll
      for (int i = 0; i < P; ++i) {
        float4 lo;
        lo.x = tf32_low(x[i].x);
        lo.y = tf32_low(x[i].y);
        lo.z = tf32_low(x[i].z);
        lo.w = tf32_low(x[i].w);
        sts4(lo_s + off[i], lo);
      }
    } else {
      const bool rows_fast = o.mode == kModeScalarR;
      for (int t = tid; t < R * 32; t += kThreads) {
        const int r = rows_fast ? t % R : t >> 5;
        const int k = rows_fast ? t / R : t & 31;
        const uint32_t off = kmajor_off(r, k);
        *reinterpret_cast<float*>(lo_gen + off) =
            tf32_low(*reinterpret_cast<const float*>(raw_gen + off));
      }
    }
  }
};

// The epilogue over up to U output elements at once. Every global load it
// needs (bias, ReLU-backward mask, the old output when accumulating) is
// issued before any store, so the U elements share one memory round trip;
// one element per iteration would serialise a round trip per element.
// Rows equal to `ex.row2` are the synthetic ones row: column sums of B,
// stored unscaled into `ex.out2`.

// One output value: alpha * acc (+ bias in the same rounding), zeroed where
// the mask is not positive, ReLU, plus the previous output.
__device__ __forceinline__ float epi_value(const ttrl_epilogue& ep, float acc, float add, float mk,
                                           float old) {
  float v = ep.bias_mode != TTRL_BIAS_NONE ? __fmaf_rn(ep.alpha, acc, add)
                                           : __fmul_rn(ep.alpha, acc);
  if (!(mk > 0.f)) v = 0.f;
  if (ep.relu) v = v > 0.f ? v : 0.f;
  if (ep.accumulate) v = __fadd_rn(v, old);
  return v;
}

template <int U>
__device__ __forceinline__ void epi_store_batch(const ttrl_epilogue& ep, const EpiExtra& ex,
                                                const int (&r)[U], const int (&c)[U],
                                                const float (&acc)[U], int n) {
  float add[U], mk[U], old[U];
  long long oo[U], mo[U];  // output and mask offsets of each element
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (ex.scatter_s) {
      const int q = fdiv(ex.f_sc, c[u]);
      const int ch = c[u] - q * ex.scatter_c;
      const int py = fdiv(ex.f_s, q);
      const int px = q - py * ex.scatter_s;
      const int img = fdiv(ex.f_ghw, r[u]);
      const int rem = r[u] - img * ex.scatter_gh * ex.scatter_gw;
      const int i = fdiv(ex.f_gw, rem);
      const int j = rem - i * ex.scatter_gw;
      const long long pix =
          (static_cast<long long>(img) * ex.scatter_h + ex.scatter_s * i + py) * ex.scatter_w +
          ex.scatter_s * j + px;
      oo[u] = pix * ep.ors + static_cast<long long>(ch) * ep.ocs;
      mo[u] = pix * ep.mrs + static_cast<long long>(ch) * ep.mcs;
    } else {
      oo[u] = static_cast<long long>(r[u]) * ep.ors + static_cast<long long>(c[u]) * ep.ocs;
      mo[u] = static_cast<long long>(r[u]) * ep.mrs + static_cast<long long>(c[u]) * ep.mcs;
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    add[u] = 0.f;
    mk[u] = 1.f;
    old[u] = 0.f;
    if (u < n) {
      if (ex.row2 >= 0 && r[u] == ex.row2) {
        if (ex.accumulate2) old[u] = ex.out2[static_cast<long long>(c[u]) * ex.cs2];
      } else {
        if (ep.bias_mode == TTRL_BIAS_ROW) {
          add[u] = ep.bias[r[u]];
        } else if (ep.bias_mode == TTRL_BIAS_COL) {
          add[u] = ep.bias[c[u]];
        }
        if (ep.mask != nullptr) mk[u] = ep.mask[mo[u]];
        if (ep.accumulate) old[u] = ep.out[oo[u]];
      }
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (u >= n) continue;
    if (ex.row2 >= 0 && r[u] == ex.row2) {
      float v = acc[u];
      if (ex.accumulate2) v += old[u];
      ex.out2[static_cast<long long>(c[u]) * ex.cs2] = v;
      continue;
    }
    ep.out[oo[u]] = epi_value(ep, acc[u], add[u], mk[u], old[u]);
  }
}


__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Staged accumulator tile in shared memory. Its layout follows the output's
// contiguous dimension so the stores coalesce and the cluster reduction can
// move 16-byte groups: row-major (column fastest, row pitch BN + 4 floats)
// for ordinary outputs, column-major (row fastest, column pitch 132) for
// transposed ones (ors == 1). The +4 padding keeps 16-byte alignment and
// spreads the per-row writes from TMEM over the banks.
template <int BN>
struct Stage {
  static constexpr int kLdRow = BN + 4;
  static constexpr int kLdCol = 128 + 4;
  static constexpr int kBytes = (128 * kLdRow > BN * kLdCol ? 128 * kLdRow : BN * kLdCol) * 4;
};

__device__ __forceinline__ float4 ld_smem4(uint32_t saddr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(saddr));
  return v;
}

// 16 bytes of shared memory at `saddr` in cluster CTA `rank` (DSMEM).
__device__ __forceinline__ float4 ld_dsmem4(uint32_t saddr, int rank) {
  uint32_t remote;
  float4 v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(saddr), "r"(rank));
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote));
  return v;
}

__device__ __forceinline__ bool aligned16_dev(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Whether groups of 4 consecutive elements along the staged tile's
// contiguous dimension are 4 consecutive, 16-byte aligned floats of the
// output (and of the mask): then the epilogue moves them as float4.
__device__ __forceinline__ bool epi_vec_ok(const ttrl_epilogue& ep, const EpiExtra& ex,
                                           bool colmajor) {
  if (!aligned16_dev(ep.out)) return false;
  if (!colmajor) {
    if (ep.ocs != 1 || (ep.ors & 3)) return false;
    if (ex.scatter_s && (ex.scatter_c & 3)) return false;
    if (ep.mask && (ep.mcs != 1 || (ep.mrs & 3) || !aligned16_dev(ep.mask))) return false;
  } else {
    if (ex.scatter_s || ep.ors != 1 || (ep.ocs & 3)) return false;
    if (ep.mask && (ep.mrs != 1 || (ep.mcs & 3) || !aligned16_dev(ep.mask))) return false;
  }
  return true;
}

// Up to P groups of 4 output elements, each a float4 at out + oo[p] with
// its mask at mask + mo[p] and its bias values b[p]: every mask and
// accumulate load is issued before the first store.
template <int P>
__device__ __forceinline__ void epi_store_vec(const ttrl_epilogue& ep, const long long (&oo)[P],
                                              const long long (&mo)[P], float4 bconst,
                                              const float (&bslot)[P], bool per_slot,
                                              const float4 (&acc)[P], const bool (&ok)[P]) {
  float4 mk[P], old[P];
#pragma unroll
  for (int p = 0; p < P; ++p) {
    mk[p] = make_float4(1.f, 1.f, 1.f, 1.f);
    old[p] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok[p]) {
      if (ep.mask != nullptr) mk[p] = *reinterpret_cast<const float4*>(ep.mask + mo[p]);
      if (ep.accumulate) old[p] = *reinterpret_cast<const float4*>(ep.out + oo[p]);
    }
  }
#pragma unroll
  for (int p = 0; p < P; ++p) {
    if (!ok[p]) continue;
    const float4 b = per_slot ? make_float4(bslot[p], bslot[p], bslot[p], bslot[p]) : bconst;
    float4 v;
    v.x = epi_value(ep, acc[p].x, b.x, mk[p].x, old[p].x);
    v.y = epi_value(ep, acc[p].y, b.y, mk[p].y, old[p].y);
    v.z = epi_value(ep, acc[p].z, b.z, mk[p].z, old[p].z);
    v.w = epi_value(ep, acc[p].w, b.w, mk[p].w, old[p].w);
    *reinterpret_cast<float4*>(ep.out + oo[p]) = v;
  }
}

// Staged float4 at shared byte address `off`: this CTA's, or with nsrc > 1
// the sum in cluster-rank order of the nsrc cluster CTAs' values there.
__device__ __forceinline__ float4 staged4(uint32_t off, int nsrc) {
  if (nsrc == 1) return ld_smem4(off);
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int q = 0; q < nsrc; ++q) {
    const float4 p = ld_dsmem4(off, q);
    v.x += p.x;
    v.y += p.y;
    v.z += p.z;
    v.w += p.w;
  }
  return v;
}

// Stores rows [r_lo, r_hi) x [0, cols) of a staged tile through the
// epilogue. With nsrc > 1 each value is the sum, in cluster-rank order, of
// the same element of the nsrc cluster CTAs' staged tiles. Every thread
// owns 4-element groups along the staged tile's contiguous dimension. Where
// the output layout allows (epi_vec_ok) a group moves as one float4 and P
// groups are processed together, their loads issued before any store;
// other groups (a ragged edge, the column-sum row) take the per-element
// path.
template <int BN, int P>
__device__ __forceinline__ void store_tile(const ttrl_epilogue& ep, const EpiExtra& ex,
                                           uint32_t tile_s, bool colmajor, int row0, int col0,
                                           int r_lo, int r_hi, int cols, int nsrc, int tid) {
  using St = Stage<BN>;
  const bool vec = epi_vec_ok(ep, ex, colmajor);
  int rr[4], cc[4];
  float acc[4];
  float4 vacc[P];
  float bslot[P];
  long long oo[P], mo[P];
  if (!colmajor) {
    constexpr int G = BN / 4;             // column groups per row
    constexpr int RSTEP = kThreads / G;   // rows per pass
    const int c0 = (tid % G) * 4;
    if (c0 >= cols) return;
    const bool full = vec && c0 + 4 <= cols;
    const int col = col0 + c0;
    // Per-thread constants of the group's columns: their bias values and,
    // for a sub-pixel scatter, their parity class and first channel.
    float4 bcol = make_float4(0.f, 0.f, 0.f, 0.f);
    if (full && ep.bias_mode == TTRL_BIAS_COL)
      bcol = make_float4(ep.bias[col], ep.bias[col + 1], ep.bias[col + 2], ep.bias[col + 3]);
    int ch = col, py = 0, px = 0;
    if (full && ex.scatter_s) {
      const int q = fdiv(ex.f_sc, col);
      ch = col - q * ex.scatter_c;
      py = fdiv(ex.f_s, q);
      px = q - py * ex.scatter_s;
    }
    for (int rb = r_lo + tid / G; rb < r_hi; rb += RSTEP * P) {
      bool ok[P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        ok[p] = false;
        oo[p] = mo[p] = 0;
        const int r = rb + p * RSTEP;
        if (r >= r_hi) continue;
        const float4 v = staged4(tile_s + (r * St::kLdRow + c0) * 4, nsrc);
        const int row = row0 + r;
        if (!full || row == ex.row2) {
          acc[0] = v.x;
          acc[1] = v.y;
          acc[2] = v.z;
          acc[3] = v.w;
          int nv = 0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            rr[u] = row;
            cc[u] = col + u;
            if (c0 + u < cols) nv = u + 1;
          }
          epi_store_batch<4>(ep, ex, rr, cc, acc, nv);
          continue;
        }
        long long pix = row;
        if (ex.scatter_s) {
          const int img = fdiv(ex.f_ghw, row);
          const int rem = row - img * ex.scatter_gh * ex.scatter_gw;
          const int i = fdiv(ex.f_gw, rem);
          const int j = rem - i * ex.scatter_gw;
          pix = (static_cast<long long>(img) * ex.scatter_h + ex.scatter_s * i + py) *
                    ex.scatter_w + ex.scatter_s * j + px;
        }
        oo[p] = pix * ep.ors + ch;
        mo[p] = pix * ep.mrs + ch;
        vacc[p] = v;
        bslot[p] = ep.bias_mode == TTRL_BIAS_ROW ? ep.bias[row] : 0.f;
        ok[p] = true;
      }
      epi_store_vec<P>(ep, oo, mo, bcol, bslot, ep.bias_mode == TTRL_BIAS_ROW, vacc, ok);
    }
  } else {
    const int r_span = r_hi - r_lo;
    const int G = (r_span + 3) / 4;       // row groups in the slice (<= 32)
    const int rg = tid & 31;
    if (rg >= G) return;
    const int r = r_lo + rg * 4;
    const int row = row0 + r;
    const bool full = vec && r + 4 <= r_hi && !(ex.row2 >= row && ex.row2 < row + 4);
    float4 brow = make_float4(0.f, 0.f, 0.f, 0.f);
    if (full && ep.bias_mode == TTRL_BIAS_ROW)
      brow = make_float4(ep.bias[row], ep.bias[row + 1], ep.bias[row + 2], ep.bias[row + 3]);
    for (int cb = tid >> 5; cb < cols; cb += (kThreads / 32) * P) {
      bool ok[P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        ok[p] = false;
        oo[p] = mo[p] = 0;
        const int c = cb + p * (kThreads / 32);
        if (c >= cols) continue;
        const float4 v = staged4(tile_s + (c * St::kLdCol + r) * 4, nsrc);
        if (!full) {
          acc[0] = v.x;
          acc[1] = v.y;
          acc[2] = v.z;
          acc[3] = v.w;
          int nv = 0;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            rr[u] = row + u;
            cc[u] = col0 + c;
            if (r + u < r_hi) nv = u + 1;
          }
          epi_store_batch<4>(ep, ex, rr, cc, acc, nv);
          continue;
        }
        const long long colv = col0 + c;
        oo[p] = row + colv * ep.ocs;
        mo[p] = row + colv * ep.mcs;
        vacc[p] = v;
        bslot[p] = ep.bias_mode == TTRL_BIAS_COL ? ep.bias[colv] : 0.f;
        ok[p] = true;
      }
      epi_store_vec<P>(ep, oo, mo, brow, bslot, ep.bias_mode == TTRL_BIAS_COL, vacc, ok);
    }
  }
}

// Long-K split through global memory: the last split CTA of a tile sums
// the partial planes in split order (loads batched over planes and
// elements) and applies the epilogue.
template <int BN>
__device__ __forceinline__ void reduce_partials(const ttrl_epilogue& ep, const EpiExtra& ex,
                                                const float* ws, int m, int n, int row0, int col0,
                                                int rows, int cols, int tid) {
  const long long plane = static_cast<long long>(m) * n;
  const int zs = static_cast<int>(gridDim.z);
  constexpr int U = 4, Z = 4;
  constexpr int RSTEP = kThreads / BN;
  const int c = tid & (BN - 1);
  if (c >= cols) return;
  for (int rb = tid / BN; rb < rows; rb += RSTEP * U) {
    int rr[U], cc[U];
    float sum[U];
    int nv = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      rr[u] = row0 + rb + u * RSTEP;
      cc[u] = col0 + c;
      sum[u] = 0.f;
      if (rb + u * RSTEP < rows) nv = u + 1;
    }
    for (int z0 = 0; z0 < zs; z0 += Z) {
      float p[Z][U];
#pragma unroll
      for (int z = 0; z < Z; ++z)
#pragma unroll
        for (int u = 0; u < U; ++u)
          p[z][u] = (z0 + z < zs && u < nv)
                        ? __ldcg(ws + (z0 + z) * plane + static_cast<long long>(rr[u]) * n + cc[u])
                        : 0.f;
#pragma unroll
      for (int z = 0; z < Z; ++z)
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (z0 + z < zs) sum[u] += p[z][u];
    }
    epi_store_batch<U>(ep, ex, rr, cc, sum, nv);
  }
}

// One operand tile of R rows x 32 k by TMA, into the same shared-memory
// layout the cp.async gathers produce: K-major tiles as one box (128-byte
// swizzle), MN-major tiles as R/32 boxes of 32 rows x 32 k (128-byte swizzle
// with 32-byte atoms). Coordinates are innermost first; the innermost one is
// a multiple of 4 floats (16 bytes) by construction.
template <int R>
__device__ __forceinline__ void tma_operand(const CUtensorMap* map, bool mn, uint32_t dst,
                                            int row0, int k0, uint32_t bar) {
  if (!mn) {
    tma_load_2d(dst, map, k0, row0, bar);
  } else {
#pragma unroll
    for (int g = 0; g < R / 32; ++g) tma_load_2d(dst + g * 4096, map, row0 + g * 32, k0, bar);
  }
}

// Window origin (input column, input row, image) of output pixel `p` of a
// convolution operand.
struct WindowOrigin {
  int w, h, n;
};
__device__ __forceinline__ WindowOrigin window_origin(const DevOperand& o, int p) {
  const int img = fdiv(o.f_ohw, p);
  const int rem = p - img * o.oh * o.ow;
  const int oy = fdiv(o.f_ow, rem);
  const int ox = rem - oy * o.ow;
  return {ox * o.stride - o.pad, oy * o.stride - o.pad, img};
}

// One stage of a convolution operand by TMA im2col mode. The map's pixel
// box is 32 channels, so each load covers one filter tap (C is a multiple of
// 32 whenever this path is taken).
//  - conv fprop windows (K-major): 128 output pixels from `row0`, reduction
//    columns k0 .. k0+31 = tap k0 / C, channels k0 % C .. +31.
//  - weight-gradient windows (MN-major): R rows of (tap, channel) from
//    `row0` in groups of 32, each group the 32 pixels k0 .. k0+31 of one
//    tap; groups past the last row repeat the last tap (those rows of D are
//    never stored; the bias gradient's ones row is written over them).
template <int R>
__device__ __forceinline__ void tma_im2col_operand(const CUtensorMap* map, const DevOperand& o,
                                                   bool mn, uint32_t dst, int row0, int k0,
                                                   uint32_t bar) {
  if (!mn) {
    const WindowOrigin wo = window_origin(o, row0);
    const int t = fdiv(o.f_c, k0);
    const int ky = fdiv(o.f_kw, t);
    tma_load_im2col_4d(dst, map, k0 - t * o.c, wo.w, wo.h, wo.n,
                       static_cast<uint16_t>(t - ky * o.kw), static_cast<uint16_t>(ky), bar);
  } else {
    const WindowOrigin wo = window_origin(o, k0);
    const int last = o.kh * o.kw - 1;
#pragma unroll
    for (int g = 0; g < R / 32; ++g) {
      const int r = row0 + g * 32;
      int t = fdiv(o.f_c, r);
      const int c = r - t * o.c;
      if (t > last) t = last;
      const int ky = fdiv(o.f_kw, t);
      tma_load_im2col_4d(dst + g * 4096, map, c, wo.w, wo.h, wo.n,
                         static_cast<uint16_t>(t - ky * o.kw), static_cast<uint16_t>(ky), bar);
    }
  }
}

// SMALL: a half-size footprint (about 100 KB of shared memory, <= 102
// registers) so two CTAs share an SM; used for grids of several waves, where
// one CTA's set-up, pipeline fill and epilogue overlap the other's main loop.
template <int BN, bool SPLIT, bool SMALL>
struct TileCfg {
  static constexpr int kABytes = 128 * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kTile = kABytes + kBBytes;  // one raw (or lo) stage
  // Split-TF32 keeps the low parts in a ring of their own, freed by the MMA
  // commits, so neither ring waits on the other's round trip.
  static constexpr int kLoSlots =
      !SPLIT ? 0 : SMALL ? (BN >= 128 ? 1 : 2) : (BN >= 128 ? 3 : 4);
  static constexpr int kBudget = (SMALL ? 100 : 196) * 1024 - kLoSlots * kTile;
  static constexpr int kRawFit = kBudget / kTile;
  static constexpr int kStages = kRawFit > 8 ? 8 : kRawFit;
  // Gathered (cp.async) operands refill a raw stage once the MMAs of the
  // k-block two iterations back have drained; TMA operands are refilled by
  // the producer warp as soon as a stage drains.
  static constexpr int kLag = kStages >= 4 ? 2 : 1;
  static constexpr int kAhead = kStages - kLag;  // k-blocks in flight
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem =
      (kStages + kLoSlots) * kTile + 1024 /*align slack*/ + 512 /*barriers*/;
  static_assert(kStages >= 2, "at least two pipeline stages");
  // With both operands by TMA, the two loader groups take alternate k-blocks
  // and the first kStages of them land without any MMA having run, so a
  // loader can reach k-block i when only the MMAs of k-block i - kStages
  // are known to be done. Its wait for low-part slot i % kLoSlots is a
  // parity wait on the MMAs of k-block i - kLoSlots; it is only sound when
  // the slot's previous phase (k-block i - 2 kLoSlots) is already complete,
  // or a wait one phase early passes at once and the loader overwrites low
  // parts the MMAs still read.
  static_assert(!SPLIT || kStages <= 2 * kLoSlots,
                "a loader may run at most one low-part-slot phase ahead of the MMAs");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
  static_assert((kStages + kLoSlots) * kTile >= Stage<BN>::kBytes,
                "epilogue staging fits in the rings");
};

// Named barrier over the 256 loader threads (the MMA warp does not join).
__device__ __forceinline__ void loader_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
}

template <int BN, bool SPLIT, bool SMALL>
__global__ void __launch_bounds__(kBlockThreads, SMALL ? 2 : 1)
    gemm_tc_kernel(const __grid_constant__ GemmArgs args) {
  using Cfg = TileCfg<BN, SPLIT, SMALL>;
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
  const uint32_t tfull0 = loempty0 + (L > 0 ? L : 1) * 8;  // S "TMA bytes landed"
  const uint32_t accum_bar = tfull0 + S * 8;
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
  if (warp == kProducerWarp && lane == 0) {
    // The descriptors are launch parameters, so their fetch can overlap the
    // previous kernel's tail.
    if (args.a_tma) prefetch_tensormap(&args.tma_a);
    if (args.b_tma) prefetch_tensormap(&args.tma_b);
  }
  // Both operands by TMA: the loader warps work in groups (see kLoaderGroups).
  const bool grouped = args.a_tma != 0 && args.b_tma != 0;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(empty0 + s * 8, 1);
      mbar_init(full0 + s * 8, grouped ? kGroupWarps : kLoadWarps);
      mbar_init(tfull0 + s * 8, 1);
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
  const bool round_a = !SPLIT && !args.a.exact;
  const bool round_b = !SPLIT && !args.b.exact;
  bool timed_out = false;

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_gen;
  // Set-up above touched no global memory; from here on the previous
  // kernel's results are read and this kernel's outputs written.
  pdl_trigger();
  pdl_wait();

  auto raw_a = [&](int s) { return sbase + s * Cfg::kTile; };
  auto raw_b = [&](int s) { return sbase + s * Cfg::kTile + Cfg::kABytes; };

  if (warp < kLoadWarps) {
    // ---- loader warps ----
    // Operand descriptors in registers: helpers that read them through a
    // reference to the kernel parameter block would reload every field
    // (a generic load) after each copy instruction.
    const DevOperand oa = args.a;
    const DevOperand ob = args.b;
    Loader<128> la;
    Loader<BN> lb;
    la.init(oa, row0, tid);
    lb.init(ob, col0, tid);
    // Dense operands arrive by TMA (the producer warp issues each stage and
    // the bytes complete on tfull); gathered ones by per-thread cp.async.
    const bool a_tma = args.a_tma != 0, b_tma = args.b_tma != 0;
    const bool any_tma = a_tma || b_tma;
    const bool any_gather = !(a_tma && b_tma);
    // An MN-major A loaded by TMA (dense, or a weight gradient's windows)
    // whose appended ones row is not in memory: the TMA fills it with zeros
    // and the loader warps write the ones into each stage after it lands.
    const bool a_ones_by_loader = a_tma && a_mn && oa.ones_row;
    auto issue_gathers = [&](int st, int kb) {
      const int k0 = kb * 32;
      if (!a_tma) la.issue(oa, raw_a(st), row0, k0, tid);
      if (!b_tma) lb.issue(ob, raw_b(st), col0, k0, tid);
    };
    if (grouped) {
      // Group g takes k-blocks g, g + kLoaderGroups, ...; each thread covers
      // kLoaderGroups thread slots of the 256-thread stage layout.
      const int grp = warp / kGroupWarps;
      const int gt = tid % kGroupThreads;
#pragma unroll 1
      for (int i = grp; i < nk; i += kLoaderGroups) {
        const int s = i % S;
        if (!mbar_wait(tfull0 + s * 8, (i / S) & 1)) timed_out = true;
#pragma unroll
        for (int v = 0; v < kLoaderGroups; ++v) {
          const int vt = gt + v * kGroupThreads;
          if (a_ones_by_loader)
            la.fill_ones_row(oa, sgen + s * Cfg::kTile, row0, (kb0 + i) * 32, vt);
          if (round_a) la.round_in_place(oa, sgen + s * Cfg::kTile, raw_a(s), vt);
          if (round_b)
            lb.round_in_place(ob, sgen + s * Cfg::kTile + Cfg::kABytes, raw_b(s), vt);
        }
        if (split_a || split_b) {
          const int l = i % LL;
          if (i >= L && !mbar_wait(loempty0 + l * 8, ((i - L) / LL) & 1)) timed_out = true;
          const uint8_t* hi = sgen + s * Cfg::kTile;
          uint8_t* lo = sgen + (lo_base - sbase) + l * Cfg::kTile;
          const uint32_t lo_s = lo_base + l * Cfg::kTile;
#pragma unroll
          for (int v = 0; v < kLoaderGroups; ++v) {
            const int vt = gt + v * kGroupThreads;
            if (split_a) la.split(oa, hi, lo, raw_a(s), lo_s, vt);
            if (split_b)
              lb.split(ob, hi + Cfg::kABytes, lo + Cfg::kABytes, raw_b(s), lo_s + Cfg::kABytes,
                       vt);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(full0 + s * 8);
      }
    }
    if (any_gather) {
#pragma unroll 1
      for (int s = 0; s < AHEAD; ++s) {
        if (s < nk) issue_gathers(s, kb0 + s);
        cp_async_commit();
      }
    }
#pragma unroll 1
    for (int i = 0; i < (grouped ? 0 : nk); ++i) {
      if (any_gather) {
        const int j = i + AHEAD;
        if (j < nk) {
          const int sj = j % S;
          if (j >= S) {
            // Raw stage sj was last read by the MMAs of k-block j - S.
            if (!mbar_wait(empty0 + sj * 8, ((j - S) / S) & 1)) timed_out = true;
          }
          issue_gathers(sj, kb0 + j);
        }
        cp_async_commit();
        cp_async_wait<AHEAD>();  // this thread's copies of k-block i have landed
      }
      const int s = i % S;
      if (any_tma && !mbar_wait(tfull0 + s * 8, (i / S) & 1)) timed_out = true;
      if (a_ones_by_loader) la.fill_ones_row(oa, sgen + s * Cfg::kTile, row0, (kb0 + i) * 32, tid);
      if (round_a) la.round_in_place(oa, sgen + s * Cfg::kTile, raw_a(s), tid);
      if (round_b)
        lb.round_in_place(ob, sgen + s * Cfg::kTile + Cfg::kABytes, raw_b(s), tid);
      if (split_a || split_b) {
        const int l = i % LL;
        if (i >= L) {
          // Lo slot l was last read by the MMAs of k-block i - L.
          if (!mbar_wait(loempty0 + l * 8, ((i - L) / LL) & 1)) timed_out = true;
        }
        const uint8_t* hi = sgen + s * Cfg::kTile;
        uint8_t* lo = sgen + (lo_base - sbase) + l * Cfg::kTile;
        const uint32_t lo_s = lo_base + l * Cfg::kTile;
        if (split_a) la.split(oa, hi, lo, raw_a(s), lo_s, tid);
        if (split_b)
          lb.split(ob, hi + Cfg::kABytes, lo + Cfg::kABytes, raw_b(s), lo_s + Cfg::kABytes, tid);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(full0 + s * 8);
    }
  } else if (warp == kProducerWarp) {
    // ---- TMA producer: refills each raw stage as soon as its MMAs drain ----
    const bool a_tma = args.a_tma != 0, b_tma = args.b_tma != 0;
    if ((a_tma || b_tma) && lane == 0) {
      const uint32_t tma_bytes = (a_tma ? Cfg::kABytes : 0) + (b_tma ? Cfg::kBBytes : 0);
#pragma unroll 1
      for (int j = 0; j < nk; ++j) {
        const int st = j % S;
        if (j >= S) {
          if (!mbar_wait(empty0 + st * 8, ((j - S) / S) & 1)) timed_out = true;
        }
        const int k0 = (kb0 + j) * 32;
        mbar_arrive_expect_tx(tfull0 + st * 8, tma_bytes);
        if (a_tma) {
          if (args.im2col & 1)
            tma_im2col_operand<128>(&args.tma_a, args.a, a_mn, raw_a(st), row0, k0,
                                    tfull0 + st * 8);
          else
            tma_operand<128>(&args.tma_a, a_mn, raw_a(st), row0, k0, tfull0 + st * 8);
        }
        if (b_tma) {
          if (args.im2col & 2)
            tma_im2col_operand<BN>(&args.tma_b, args.b, b_mn, raw_b(st), col0, k0,
                                   tfull0 + st * 8);
          else
            tma_operand<BN>(&args.tma_b, b_mn, raw_b(st), col0, k0, tfull0 + st * 8);
        }
      }
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

  // ---- epilogue: TMEM -> registers -> staged tile in shared memory (the
  // ring is idle once the accumulator is ready, so the tile reuses it) ----
  const int rows = min(128, args.m - row0);
  const int cols = min(BN, args.n - col0);
  float* tile = reinterpret_cast<float*>(sgen);
  const bool colmajor = args.ep.ors == 1 && args.ep.ocs != 1 && args.ws == nullptr;
  if (warp < kLoadWarps) {
    if (!mbar_wait(accum_bar, 0)) timed_out = true;
    tc_fence_after();
    const int rl = (warp & 3) * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int cbeg = (warp >> 2) * (BN / 2);
#pragma unroll 1
    for (int c = cbeg; c < cbeg + BN / 2; c += 8) {
      if (c >= cols) break;  // uniform across the warp
      float v[8];
      tmem_ld8(trow + c, v);
      if (!colmajor) {
        float4* dst = reinterpret_cast<float4*>(tile + rl * Stage<BN>::kLdRow + c);
        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) tile[(c + q) * Stage<BN>::kLdCol + rl] = v[q];
      }
    }
  }
  tc_fence_before();
  __syncthreads();  // the staged tile is complete and TMEM is no longer read
  if (warp == kMmaWarp) tmem_dealloc(tmem, Cfg::kTmemCols);
  if (timed_out) record_error(args.status, kErrWaitTimeout);

  const int csplits = args.cluster_splits;
  const ttrl_epilogue ep = args.ep;  // in registers, see the operand copies above
  const EpiExtra ex = args.ex;
  if (csplits > 1) {
    // The split CTAs of this tile are one cluster. Once every partial is
    // staged, CTA `rank` sums rows [rank*per, (rank+1)*per) across the
    // cluster's shared memory in split order and stores them.
    cluster_sync_all();
    const int rank = static_cast<int>(cluster_ctarank());
    // Row slices in multiples of 4 so column-major groups stay aligned.
    const int per = ((rows + csplits - 1) / csplits + 3) & ~3;
    const int r_lo = min(rows, rank * per);
    const int r_hi = min(rows, r_lo + per);
    if (warp < kLoadWarps)
      store_tile<BN, SMALL ? 1 : 4>(ep, ex, smem_u32(tile), colmajor, row0, col0, r_lo, r_hi, cols, csplits,
                     tid);
    cluster_sync_all();  // peers have finished reading this CTA's tile
  } else if (warp < kLoadWarps) {
    if (args.ws == nullptr) {
      store_tile<BN, SMALL ? 1 : 4>(ep, ex, smem_u32(tile), colmajor, row0, col0, 0, rows, cols, 1, tid);
    } else {
      // Long-K split through global memory: this split's partial tile.
      float* wz = args.ws + static_cast<long long>(blockIdx.z) * args.m * args.n;
      constexpr int RSTEP = kThreads / BN;
      const int c = tid & (BN - 1);
      if (c < cols) {
#pragma unroll 4
        for (int r = tid / BN; r < rows; r += RSTEP)
          wz[static_cast<long long>(row0 + r) * args.n + col0 + c] =
              tile[r * Stage<BN>::kLdRow + c];
      }
    }
  }

  if (args.ws != nullptr && csplits <= 1 && args.reduce_in_kernel) {
    // The last split CTA of this tile sums every partial in split order.
    const int tile_id = blockIdx.y * gridDim.x + blockIdx.x;
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(reinterpret_cast<unsigned*>(args.counters) + tile_id, 1u);
      s_last = (prev == gridDim.z - 1) ? 1 : 0;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      if (warp < kLoadWarps)
        reduce_partials<BN>(ep, ex, args.ws, args.m, args.n, row0, col0, rows, cols, tid);
      if (tid == 0) args.counters[tile_id] = 0;
    }
  }
}

// Sum split-K partials in split order and apply the epilogue (used when the
// partial tiles are too large for one CTA to reduce quickly).
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int m, int n,
                                     ttrl_epilogue ep, EpiExtra ex) {
  pdl_trigger();
  pdl_wait();
  const long long total = static_cast<long long>(m) * n;
  constexpr int Z = 8;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    int r[1], c[1];
    r[0] = static_cast<int>(idx / n);
    c[0] = static_cast<int>(idx - static_cast<long long>(r[0]) * n);
    float s[1] = {0.f};
    for (int z0 = 0; z0 < splits; z0 += Z) {
      float p[Z];
#pragma unroll
      for (int z = 0; z < Z; ++z)
        p[z] = z0 + z < splits ? ws[static_cast<long long>(z0 + z) * total + idx] : 0.f;
#pragma unroll
      for (int z = 0; z < Z; ++z)
        if (z0 + z < splits) s[0] += p[z];
    }
    epi_store_batch<1>(ep, ex, r, c, s, 1);
  }
}

// ------------------------------------------------------------------ host

// Sets the kernel's shared-memory limit, allows clusters above the portable
// size 8, and returns the largest split-K cluster (16 or 8) the device can
// co-schedule at this kernel's footprint.
template <int BN, bool SPLIT>
static int set_smem_attr(int* cluster_cap) {
  using Cfg = TileCfg<BN, SPLIT, false>;
  using Small = TileCfg<BN, SPLIT, true>;
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, SPLIT, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(gemm)", e);
  e = cudaFuncSetAttribute(gemm_tc_kernel<BN, SPLIT, true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, Small::kSmem);
  if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(gemm, small)", e);
  int cap = 8;
  if (cudaFuncSetAttribute(gemm_tc_kernel<BN, SPLIT, false>,
                           cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, 16);
    cfg.blockDim = dim3(kBlockThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 16;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_tc_kernel<BN, SPLIT, false>, &cfg) ==
            cudaSuccess &&
        clusters >= 1)
      cap = 16;
  }
  cudaGetLastError();  // a refused probe leaves no sticky error
  if (cap < *cluster_cap) *cluster_cap = cap;
  return TTRL_OK;
}

// Records g_active_clusters for one variant (cudaOccupancyMaxActiveClusters
// over cluster sizes 2..cap: clusters pack into GPCs, so fewer of a size
// that does not divide a GPC's SMs fit than the SM count suggests).
template <int BN, bool SPLIT>
static void record_active_clusters(int dev, int cap) {
  using Cfg = TileCfg<BN, SPLIT, false>;
  const int bi = BN == 32 ? 0 : BN == 64 ? 1 : 2;
  for (int cz = 2; cz <= cap && cz <= 16; ++cz) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, cz);
    cfg.blockDim = dim3(kBlockThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = cz;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_tc_kernel<BN, SPLIT, false>, &cfg) ==
        cudaSuccess)
      g_active_clusters[dev][bi][SPLIT ? 1 : 0][cz] = clusters;
  }
  cudaGetLastError();  // a refused query leaves no sticky error
}

int gemm_init_device() {
  int rc = TTRL_OK;
  int cap = 16;
  if ((rc = set_smem_attr<32, true>(&cap))) return rc;
  if ((rc = set_smem_attr<64, true>(&cap))) return rc;
  if ((rc = set_smem_attr<128, true>(&cap))) return rc;
  if ((rc = set_smem_attr<32, false>(&cap))) return rc;
  if ((rc = set_smem_attr<64, false>(&cap))) return rc;
  if ((rc = set_smem_attr<128, false>(&cap))) return rc;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
    g_max_cluster[dev] = cap;
    record_active_clusters<32, true>(dev, cap);
    record_active_clusters<64, true>(dev, cap);
    record_active_clusters<128, true>(dev, cap);
    record_active_clusters<32, false>(dev, cap);
    record_active_clusters<64, false>(dev, cap);
    record_active_clusters<128, false>(dev, cap);
  }
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

// cuTensorMapEncodeTiled, fetched once through the runtime (no link against
// the driver library).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

// cuTensorMapEncodeIm2col, fetched the same way.
static PFN_cuTensorMapEncodeIm2col_v12000 im2col_map_encoder() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

// Convolution operands whose windows TMA im2col mode loads (bit 0: conv
// fprop A, bit 1: conv wgrad B). TTRL_IM2COL_TMA overrides (0 = gather both
// with cp.async).
static int im2col_modes() {
  static int modes = [] {
    const char* e = std::getenv("TTRL_IM2COL_TMA");
    return e ? std::atoi(e) : 3;
  }();
  return modes;
}

// The im2col TMA map of a convolution operand (NHWC activation, C a multiple
// of 32): pixel box of 32 channels; 128 pixels per load for fprop's windows
// (one K-major stage), 32 for the weight gradient's (one 32-row group of an
// MN-major stage); bounding box of window origins
// [-pad, extent - 1 + pad - (kernel - 1)] walked with the conv stride. False
// when the operand does not qualify (it is then gathered).
static bool encode_im2col_map(const DevOperand& o, CUtensorMap* map) {
  const bool fprop = o.kind == TTRL_OPND_CONV_FPROP && o.mode == kModeKVec && !o.ones_row;
  // A weight gradient's windows operand may carry the ones row of the bias
  // gradient: the loader warps write it into each stage after the TMA lands.
  const bool wgrad = o.kind == TTRL_OPND_CONV_WGRAD && o.mode == kModeMNVec;
  if (!(fprop && (im2col_modes() & 1)) && !(wgrad && (im2col_modes() & 2))) return false;
  const int pixels = fprop ? 128 : 32;
  if (o.c % 32 != 0 || !aligned16(o.ptr)) return false;
  if (o.stride < 1 || o.stride > 8 || o.pad > 127 || o.kh != o.kw) return false;
  const int upper = o.pad - (o.kw - 1);
  if (upper < -128 || o.w + 2 * o.pad < o.kw || o.h + 2 * o.pad < o.kh) return false;
  PFN_cuTensorMapEncodeIm2col_v12000 enc = im2col_map_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(o.c), static_cast<cuuint64_t>(o.w),
                              static_cast<cuuint64_t>(o.h), static_cast<cuuint64_t>(o.n)};
  const cuuint64_t row = static_cast<cuuint64_t>(o.c) * 4;
  const cuuint64_t strides[3] = {row, row * o.w, row * o.w * o.h};
  if (strides[2] >= (1ull << 40)) return false;
  const int lower_corner[2] = {-o.pad, -o.pad};
  const int upper_corner[2] = {upper, upper};
  const cuuint32_t es[4] = {1, static_cast<cuuint32_t>(o.stride),
                            static_cast<cuuint32_t>(o.stride), 1};
  const CUtensorMapSwizzle sw =
      fprop ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  const CUresult r =
      enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(o.ptr), dims, strides,
          lower_corner, upper_corner, 32, static_cast<cuuint32_t>(pixels), es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The TMA map of a dense operand whose tiles are R rows x 32 k, or false
// when the operand is gathered instead (conv windows, odd strides or
// alignment, or an appended ones row of a K-major operand).
static bool encode_operand_map(const DevOperand& o, int R, CUtensorMap* map) {
  if (o.kind != TTRL_OPND_DENSE) return false;
  // An appended ones row (the bias gradient's) lies past the map's extent in
  // MN-major tiles, where the TMA writes zeros and the loader warps the ones.
  if (o.ones_row && o.mode != kModeMNVec) return false;
  if (o.mode != kModeKVec && o.mode != kModeMNVec) return false;
  if (o.rows <= 0 || o.kdim <= 0) return false;
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t dims[2];
  cuuint64_t strides[1];
  cuuint32_t box[2];
  const cuuint32_t es[2] = {1, 1};
  CUtensorMapSwizzle sw;
  if (o.mode == kModeKVec) {  // rows of K contiguous floats
    dims[0] = static_cast<cuuint64_t>(o.kdim);
    dims[1] = static_cast<cuuint64_t>(o.rows);
    strides[0] = static_cast<cuuint64_t>(o.rs) * 4;
    box[0] = 32;
    box[1] = static_cast<cuuint32_t>(R);
    sw = CU_TENSOR_MAP_SWIZZLE_128B;
  } else {  // k lines of contiguous rows
    dims[0] = static_cast<cuuint64_t>(o.rows);
    dims[1] = static_cast<cuuint64_t>(o.kdim);
    strides[0] = static_cast<cuuint64_t>(o.ks) * 4;
    box[0] = 32;
    box[1] = 32;
    sw = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  }
  if (strides[0] % 16 != 0 || strides[0] >= (1ull << 40)) return false;
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(o.ptr), dims,
                         strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

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

// The operand resolution and TMA map encoders, for the other kernels of
// this library that load the same operands.
int gemm_resolve_operand(const ttrl_operand& in, int ones_row, DevOperand& out) {
  return resolve_operand(in, ones_row, out);
}
bool gemm_im2col_map(const DevOperand& o, CUtensorMap* map) { return encode_im2col_map(o, map); }
bool gemm_tile_map(const DevOperand& o, int rows, CUtensorMap* map) {
  return encode_operand_map(o, rows, map);
}

static int pick_bn(int n) {
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  return 128;
}

struct Schedule {
  int bn, kblocks, splits, kb_per_split, tiles;
  bool cluster;  // the splits of a tile reduce through distributed shared memory
};

static int max_cluster_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 8;
  return g_max_cluster[dev] > 0 ? g_max_cluster[dev] : 8;
}

// Resident clusters of `cz` CTAs for this tile width and precision on the
// current device, or 0 when unknown.
static int active_clusters(int bn, bool split3, int cz) {
  int dev = 0;
  if (cz < 2 || cz > 16 || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int bi = bn == 32 ? 0 : bn == 64 ? 1 : 2;
  return g_active_clusters[dev][bi][split3 ? 1 : 0][cz];
}

// Non-cluster GEMMs whose CTAs each walk at most this many k-blocks use the
// half-footprint variant.
#ifndef TTRL_SMALL_MAX_KBLOCKS
#define TTRL_SMALL_MAX_KBLOCKS 8
#endif
constexpr int kSmallMaxKBlocks = TTRL_SMALL_MAX_KBLOCKS;

static Schedule make_schedule(const ttrl_gemm_desc& d) {
  Schedule s;
  s.bn = pick_bn(d.n);
  // A quarter wave of 128-wide tiles or less (the SAC MLP's and the batch-32
  // DQN's layers): 64-wide tiles give twice the CTAs, and their smaller
  // stages leave room for a second low-part slot, so the split pass of one
  // k-block overlaps the MMAs of the previous one. Larger grids keep the
  // 128-wide tile: with several GEMMs in flight on the launch lanes, the
  // extra CTAs cost more than they gain.
  if (s.bn == 128 && ((d.m + 127) / 128) * ((d.n + 127) / 128) <= 148 / 4) s.bn = 64;
  s.kblocks = (d.k + 31) / 32;
  s.tiles = ((d.m + 127) / 128) * ((d.n + s.bn - 1) / s.bn);
  const int cmax = max_cluster_for_current_device();
  int splits = d.splits;
  bool global_split = false;
  if (splits <= 0) {
    // Aim for about one wave of 148 SMs with a few k-blocks per CTA.
    // Up to `cmax` splits reduce inside a cluster; beyond that (where each
    // CTA of a cmax-way cluster would still walk >= 4 k-blocks: DQN's conv2
    // weight gradient, 81 k-blocks over 5 tiles) up to 64 splits reduce
    // through global memory, more CTAs with shorter walks.
    splits = 1;
    if (s.tiles < 120 && s.kblocks >= 8) {
      // Whole waves only: tiles x splits stays within the 148 SMs (one CTA
      // of this kernel fits per SM), except that a single tile may use all.
      // At least 4 k-blocks per CTA, or 2 for a short reduction (8-15
      // k-blocks: SAC's 256-wide layers, 8 k-blocks over 8 tiles, take
      // 7.5 us as 4-way clusters against 9.2 us as 2-way).
      const int want = 148 / s.tiles;
      const int most = std::max(s.kblocks / 4, std::min(s.kblocks / 2, 4));
      splits = want < most ? want : most;
      if (splits > cmax) {
        if (s.kblocks / cmax >= 4) {
          global_split = true;
          if (splits > 64) splits = 64;
        } else {
          splits = cmax;
        }
      }
      // Every cluster resident at once: clusters pack into GPCs, and a
      // size that leaves some unplaced runs a second wave (PPO's fc1
      // forward, 16 tiles: 9-way clusters 26.3 us, 6-way 17.6 us). Fall
      // back to the largest size that fits in one wave.
      if (!global_split) {
        const bool split3 = d.precision == TTRL_PREC_TF32X3;
        while (splits > 1) {
          const int fit = active_clusters(s.bn, split3, splits);
          if (fit == 0 || fit >= s.tiles) break;
          --splits;
        }
      }
      if (splits < 1) splits = 1;
    }
  } else if (splits > cmax) {
    global_split = true;
  }
  if (splits > s.kblocks) splits = s.kblocks > 0 ? s.kblocks : 1;
  s.kb_per_split = (s.kblocks + splits - 1) / splits;
  if (s.kb_per_split < 1) s.kb_per_split = 1;
  s.splits = (s.kblocks + s.kb_per_split - 1) / s.kb_per_split;
  if (s.splits < 1) s.splits = 1;
  s.cluster = s.splits > 1 && !global_split;
  return s;
}

size_t gemm_workspace_bytes(const ttrl_gemm_desc& d) {
  const Schedule s = make_schedule(d);
  if (s.splits <= 1 || s.cluster) return kCounterBytes;
  return kCounterBytes + static_cast<size_t>(s.splits) * d.m * d.n * sizeof(float);
}

template <int BN, bool SPLIT, bool SMALL>
static cudaError_t launch_bn(const GemmArgs& args, dim3 grid, int cluster_z, cudaStream_t stream) {
  using Cfg = TileCfg<BN, SPLIT, SMALL>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kBlockThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cluster_z > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = static_cast<unsigned>(cluster_z);
    cfg.numAttrs = 2;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, SPLIT, SMALL>, args);
  note_launch();
  return e;
}

// ---------------------------------------------------- small dense GEMMs
//
// Products of at most kSimtMacs multiply-adds between two dense operands
// (network heads with a handful of outputs, their gradients, narrow MLP
// layers) run on the CUDA cores: one warp per output element when the
// reduction is long (lanes take every 32nd k, then a fixed shuffle tree), one
// thread per output element when it is short. At these sizes a 128-row
// tensor-core tile is mostly padding and a launch is bound by the tcgen05
// pipeline's fixed latency (TMA load, MMA, commit, TMEM read-back), not by
// math. Only when the caller lets the library choose the schedule
// (desc.splits == 0). fp32 fused multiply-adds in a fixed order: results are
// deterministic and at least as accurate as split-TF32.
constexpr long long kSimtMacs = 1ll << 20;
constexpr int kSimtWarpK = 64;  // reductions at least this long get a warp per output
constexpr int kSimtBatch = 8;   // reduction steps whose loads are issued together

struct SimtArgs {
  DevOperand a, b;
  ttrl_epilogue ep;
  EpiExtra ex;
  int32_t m, n, k;
  int32_t warp_per_output;
  int32_t c_fast;  // consecutive threads take consecutive columns (else rows)
};

__device__ __forceinline__ float simt_a(const DevOperand& o, int r, int k) {
  if (o.ones_row && r == o.rows) return 1.f;
  return o.ptr[static_cast<long long>(r) * o.rs + static_cast<long long>(k) * o.ks];
}

__global__ void __launch_bounds__(256) gemm_simt_kernel(const __grid_constant__ SimtArgs p) {
  pdl_trigger();
  pdl_wait();
  const DevOperand a = p.a, b = p.b;
  const long long outs = static_cast<long long>(p.m) * p.n;
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  long long o;
  int lane = 0;
  if (p.warp_per_output) {
    o = gid >> 5;
    lane = threadIdx.x & 31;
  } else {
    o = gid;
  }
  if (o >= outs) return;  // uniform across a warp when it owns one output
  const int r = p.c_fast ? static_cast<int>(o / p.n) : static_cast<int>(o % p.m);
  const int c = p.c_fast ? static_cast<int>(o % p.n) : static_cast<int>(o / p.m);
  // The loads of kSimtBatch consecutive reduction steps are issued before
  // their multiply-adds, which stay in sequential order: one memory round
  // trip per batch instead of per step, the same result bit for bit.
  float acc = 0.f;
  const int step = p.warp_per_output ? 32 : 1;
  int k = p.warp_per_output ? lane : 0;
  for (; k + (kSimtBatch - 1) * step < p.k; k += kSimtBatch * step) {
    float av[kSimtBatch], bv[kSimtBatch];
#pragma unroll
    for (int u = 0; u < kSimtBatch; ++u) {
      av[u] = simt_a(a, r, k + u * step);
      bv[u] = simt_a(b, c, k + u * step);
    }
#pragma unroll
    for (int u = 0; u < kSimtBatch; ++u) acc = fmaf(av[u], bv[u], acc);
  }
  for (; k < p.k; k += step) acc = fmaf(simt_a(a, r, k), simt_a(b, c, k), acc);
  if (p.warp_per_output) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane != 0) return;
  }
  const int rr[1] = {r};
  const int cc[1] = {c};
  const float v[1] = {acc};
  epi_store_batch<1>(p.ep, p.ex, rr, cc, v, 1);
}

static bool simt_eligible(const ttrl_gemm_desc& d, int a_ones_row) {
  return d.splits == 0 && d.a.kind == TTRL_OPND_DENSE && d.b.kind == TTRL_OPND_DENSE &&
         static_cast<long long>(d.m) * d.n * d.k <= kSimtMacs && (a_ones_row == 0 || d.m >= 1);
}

static int simt_run(const ttrl_gemm_desc& d, const GemmArgs& g, cudaStream_t stream) {
  SimtArgs p;
  std::memset(&p, 0, sizeof(p));
  p.a = g.a;
  p.b = g.b;
  p.ep = g.ep;
  p.ex = g.ex;
  p.m = d.m;
  p.n = d.n;
  p.k = d.k;
  p.warp_per_output = d.k >= kSimtWarpK ? 1 : 0;
  p.c_fast = d.ep.ocs <= d.ep.ors ? 1 : 0;
  const long long threads = static_cast<long long>(d.m) * d.n * (p.warp_per_output ? 32 : 1);
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  const cudaError_t le = launch_pdl(gemm_simt_kernel, dim3(blocks), dim3(256), 0, stream, p);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("gemm_simt launch", e);
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
  if (simt_eligible(d, a_ones_row)) return simt_run(d, args, stream);

  const Schedule s = make_schedule(d);
  args.kblocks = s.kblocks;
  args.kb_per_split = s.kb_per_split;
  args.a_tma = encode_operand_map(args.a, 128, &args.tma_a) ? 1 : 0;
  args.b_tma = encode_operand_map(args.b, s.bn, &args.tma_b) ? 1 : 0;
  if (!args.a_tma && encode_im2col_map(args.a, &args.tma_a)) {
    args.a_tma = 1;
    args.im2col |= 1;
  }
  if (!args.b_tma && !args.b.ones_row && encode_im2col_map(args.b, &args.tma_b)) {
    args.b_tma = 1;
    args.im2col |= 2;
  }
  if (s.cluster) {
    args.cluster_splits = s.splits;
  } else if (s.splits > 1) {
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
  const int cz = s.cluster ? s.splits : 1;
  // Several waves of CTAs, or a short walk along K (where a deep ring buys
  // little): the half-size variant runs two CTAs per SM, which also lets
  // GEMMs on concurrent launch lanes share SMs.
#ifdef TTRL_GEMM_FULL_ONLY
  const bool small = false;
#else
  const bool small = !s.cluster && (static_cast<long long>(s.tiles) * s.splits > 148 ||
                                    s.kb_per_split <= kSmallMaxKBlocks);
#endif
  cudaError_t e;
#define TTRL_LAUNCH(BNV)                                                              \
  (split3 ? (small ? launch_bn<BNV, true, true>(args, grid, cz, stream)                \
                   : launch_bn<BNV, true, false>(args, grid, cz, stream))              \
          : (small ? launch_bn<BNV, false, true>(args, grid, cz, stream)               \
                   : launch_bn<BNV, false, false>(args, grid, cz, stream)))
  switch (s.bn) {
    case 32: e = TTRL_LAUNCH(32); break;
    case 64: e = TTRL_LAUNCH(64); break;
    default: e = TTRL_LAUNCH(128); break;
  }
#undef TTRL_LAUNCH
  if (e != cudaSuccess) return set_cuda_error("gemm launch", e);
  if (s.splits > 1 && !s.cluster && !args.reduce_in_kernel) {
    if (args.ws == nullptr)
      return set_error(TTRL_EUNSUPPORTED, "gemm: split-K reduce without partials");
    const long long total = static_cast<long long>(d.m) * d.n;
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > 148 * 8) blocks = 148 * 8;
    const cudaError_t le_ = launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, stream,
                                       args.ws, s.splits, d.m, d.n, d.ep, ex);
    note_launch();
    e = le_ != cudaSuccess ? le_ : cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gemm split-k reduce launch", e);
  }
  return TTRL_OK;
}

}  // namespace ttrl
