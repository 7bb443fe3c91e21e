// Host/device structures shared between the kernels and the C-ABI layer.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/ttrl_b200.h"

namespace ttrl {

// Operand gather modes (chosen on the host from strides and alignment).
enum : int32_t {
  kModeKVec = 0,     // 16-byte chunks along k; K-major shared tile
  kModeMNVec = 1,    // 16-byte chunks along rows; MN-major shared tile
  kModeScalarK = 2,  // 4-byte gathers, k fastest across threads; K-major tile
  kModeScalarR = 3   // 4-byte gathers, rows fastest across threads; K-major tile
};

// n / d by multiply-high and shift, for 0 <= n < 2^31 (Granlund-Montgomery).
struct FastDiv {
  uint32_t d, mul, shr, pad0;
};

// n / d for 0 <= n < 2^31 by multiply-shift (d from make_fastdiv).
__device__ __forceinline__ int fdiv(const FastDiv& f, int n) {
  if (f.shr == 0) return n;  // divisor 1
  const uint32_t t = __umulhi(static_cast<uint32_t>(n), f.mul);
  return static_cast<int>((t + static_cast<uint32_t>(n)) >> f.shr);
}

FastDiv make_fastdiv(int d);

struct DevOperand {
  const float* ptr;
  int32_t kind;
  int32_t mode;
  int32_t rows, kdim;
  int64_t rs, ks;
  int32_t n, h, w, c, kh, kw, stride, pad, oh, ow;
  int32_t ones_row;  // row `rows` reads as 1.0 for every valid k
  int32_t exact;     // values exactly representable in tf32: no low part
  FastDiv f_ohw, f_ow, f_c, f_kw;  // conv index decomposition
};

// Split-K tile counters live in the first kCounterBytes of every workspace
// handed to the library; they must be zero before first use and every
// kernel leaves them zero.
constexpr size_t kCounterBytes = 64 * 1024;

// Where the synthetic ones row of operand A lands (the bias gradient).
struct EpiExtra {
  int32_t row2;  // tile row holding the column sums, or -1
  int32_t accumulate2;
  float* out2;   // out2[c * cs2]
  int64_t cs2;
  // Sub-pixel scatter of a transposed convolution (the direct data
  // gradient), off when scatter_s == 0: row r = (image, i, j) of a gh x gw
  // grid and column q * sc + ch of D is pixel (image, s*i + q / s,
  // s*j + q % s) of an h x w output, channel ch; the output and mask
  // addresses are pixel * (ors | mrs) + ch * (ocs | mcs).
  int32_t scatter_s, scatter_c, scatter_h, scatter_w, scatter_gh, scatter_gw;
  FastDiv f_sc, f_s, f_gw, f_ghw;
};

struct GemmArgs {
  // TMA tile maps of the dense operands (valid when a_tma / b_tma is set);
  // first, for their 64-byte alignment.
  CUtensorMap tma_a;
  CUtensorMap tma_b;
  DevOperand a, b;
  ttrl_epilogue ep;
  EpiExtra ex;
  int32_t m, n, k;
  int32_t kblocks;
  int32_t kb_per_split;
  int32_t reduce_in_kernel;  // last split CTA sums the partials (else a second kernel)
  int32_t cluster_splits;    // > 1: the splits of a tile form a cluster and reduce in DSMEM
  int32_t a_tma, b_tma;      // the operand's stages arrive by TMA instead of cp.async
  int32_t im2col;            // bit 0: A (conv fprop windows), bit 1: B (conv wgrad
                             // windows) by TMA im2col mode rather than a tiled map
  float* ws;      // split-K partials [splits][m][n], or null
  int* counters;  // split-K arrival counter per output tile
  int* status;
};

// Launches `kernel` with programmatic stream serialization (see pdl_wait in
// common.cuh) and counts the launch.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

int set_error(int code, const char* fmt, ...);

// Host-side count of kernels this library has enqueued (graph captures
// included), for launch accounting.
void note_launch();
int set_cuda_error(const char* what, cudaError_t e);

int gemm_init_device();
int gru_init_device();
size_t gemm_workspace_bytes(const ttrl_gemm_desc& d);
int gemm_resolve_operand(const ttrl_operand& in, int ones_row, DevOperand& out);
bool gemm_im2col_map(const DevOperand& o, CUtensorMap* map);
bool gemm_tile_map(const DevOperand& o, int rows, CUtensorMap* map);

// Stream-K convolution weight gradient (wgrad_sk.cu): one CTA per SM over a
// slice of the pixels for the whole of dW, for layers whose input is exact
// in tf32 (raw frames), C a multiple of 32, Cout 32 or 64, kh*kw*C <= 256.
bool wgrad_sk_geometry(const ttrl_conv_geom* g);
bool wgrad_sk_applies(const ttrl_conv_geom* g, const float* x, const float* dy);
size_t wgrad_sk_ws(const ttrl_conv_geom* g);
int wgrad_sk_run(const float* x, const float* dy, float* dw, float* db, const ttrl_conv_geom* g,
                 float alpha, int accumulate, int accumulate_db, int precision, float* ws,
                 size_t wsb, int* status, cudaStream_t st);
// Launch one GEMM. `counters` (kCounterBytes, zeroed) and `partials` back
// a split-K schedule; both may be null when K is not split.
int gemm_run(const ttrl_gemm_desc& d, int a_ones_row, const EpiExtra& ex, int* counters,
             float* partials, size_t partial_bytes, int* status, cudaStream_t stream);

// gemm_run over one caller workspace laid out as [counters | partials].
inline int gemm_run_ws(const ttrl_gemm_desc& d, int a_ones_row, const EpiExtra& ex, float* ws,
                       size_t ws_bytes, int* status, cudaStream_t stream) {
  const bool ok = ws != nullptr && ws_bytes >= kCounterBytes;
  return gemm_run(d, a_ones_row, ex, ok ? reinterpret_cast<int*>(ws) : nullptr,
                  ok ? reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + kCounterBytes)
                     : nullptr,
                  ok ? ws_bytes - kCounterBytes : 0, status, stream);
}

// Fused DQN loss head (ttrl/algos/dqn/losses.py:77-140).
struct DqnArgs {
  const float* q;          // [B, A] online(s), requires grad
  const float* q_sel;      // [B, A] selector: online(s') (double) or target(s')
  const float* q_tgt;      // [B, A] target(s')
  const float* onehot;     // [B, A] taken actions
  const float* rewards;    // [B]
  const float* dones;      // [B]
  const float* discounts;  // [B]
  const float* next_mask;  // [B, A] or null
  const float* is_weights; // [B] or null
  float* loss;             // [1]
  float* mean_q;           // [1]
  float* td_abs;           // [B] or null
  float* dq;               // [B, A]
  int batch, actions;
  float delta;
  int accumulate;          // dq += instead of =
};

// Fused PPO objective (ttrl/algos/ppo/loss.py:42-83).
struct PpoArgs {
  const float* logits;     // [B, A]
  const float* value;      // [B]
  const int32_t* actions;  // [B]
  const float* old_logp;   // [B]
  const float* adv;        // [B]
  const float* returns;    // [B]
  const float* old_values; // [B]
  const float* valid;      // [B] or null: masked mean (recurrent path)
  float* metrics;          // [4]: loss, policy_loss, value_loss, entropy
  float* new_logp;         // [B] or null
  float* dlogits;          // [B, A]
  float* dvalue;           // [B]
  int batch, num_actions;
  float clip, vclip, vcoef, entcoef;
};

int dqn_loss(const DqnArgs& args, cudaStream_t st);
int ppo_loss(const PpoArgs& args, cudaStream_t st);

inline EpiExtra no_extra() {
  EpiExtra e;
  e.row2 = -1;
  e.accumulate2 = 0;
  e.out2 = nullptr;
  e.cs2 = 0;
  e.scatter_s = e.scatter_c = e.scatter_h = e.scatter_w = e.scatter_gh = e.scatter_gw = 0;
  e.f_sc = e.f_s = e.f_gw = e.f_ghw = FastDiv{};
  return e;
}

}  // namespace ttrl
