// extern "C" entry points of libttrl_b200.so and the per-thread error text.
#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <cstring>

#include "internal.h"

namespace ttrl {

static thread_local char g_last_error[512] = "no error";
static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int set_cuda_error(const char* what, cudaError_t e) {
  return set_error(TTRL_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Defined in the kernel translation units.
int linear_fwd(const float*, const float*, const float*, float*, int, int, int, int, int, float*,
               size_t, int*, cudaStream_t);
int linear_dgrad(const float*, const float*, const float*, float*, int, int, int, int, int,
                 float*, size_t, int*, cudaStream_t);
int linear_wgrad(const float*, const float*, float*, float*, int, int, int, int, int, int, float*,
                 size_t, int*, cudaStream_t);
int conv_fprop(const float*, const float*, const float*, float*, const ttrl_conv_geom*, float, int,
               int, float*, size_t, int*, cudaStream_t);
int conv_dgrad(const float*, const float*, const float*, float*, const ttrl_conv_geom*, int, int,
               float*, size_t, int*, cudaStream_t);
size_t conv_dgrad_ws(const ttrl_conv_geom*);
int conv_dgrad_weights(const float*, float*, const ttrl_conv_geom*, cudaStream_t);
size_t conv_dgrad_weights_bytes(const ttrl_conv_geom*);
int conv_dgrad_prepared(const float*, const float*, const float*, float*, const ttrl_conv_geom*,
                        int, int, float*, size_t, int*, cudaStream_t);
size_t conv_dgrad_prepared_ws(const ttrl_conv_geom*);
int conv_wgrad(const float*, const float*, float*, float*, const ttrl_conv_geom*, float, int, int,
               int, float*, size_t, int*, cudaStream_t);
size_t conv_wgrad_ws(const ttrl_conv_geom*);
size_t linear_wgrad_ws(int, int, int);
int u8_to_f32(const uint8_t*, const int32_t*, float*, int, int, int, int, float, cudaStream_t);
int u8_to_f32_s2d(const uint8_t*, const int32_t*, float*, int, int, int, int, int, float,
                  cudaStream_t);
int adam_step(const ttrl_adam_tensor*, int, int32_t*, int32_t*, const float*, const double*,
              double, double, double, double, double, const double*, long long, cudaStream_t);
int grad_sqnorm(const float* const*, const int64_t*, int, float*, float, void*, size_t,
                cudaStream_t);
size_t sqnorm_ws_bytes(const int64_t*, int);
int ew(int, const float*, const int64_t*, const float*, const int64_t*, float*, const int64_t*,
       int, float, cudaStream_t);
int reduce(int, const float*, float*, int64_t, int64_t, int64_t, cudaStream_t);
int copy_strided(float*, const int64_t*, const float*, const int64_t*, const int64_t*, int, int,
                 cudaStream_t);
int polyak(float*, const float*, int64_t, float, cudaStream_t);
int blend_multi(const ttrl_blend_pair*, int, int, float, cudaStream_t);
int wait_probe(int*, cudaStream_t);
int gather_rows(const void*, const int32_t*, void*, int, int, cudaStream_t);
int gather_rows_multi(const ttrl_gather_job*, int, const int32_t*, int, cudaStream_t);



}  // namespace ttrl

using namespace ttrl;

#define TTRL_STREAM(s) static_cast<cudaStream_t>(s)

extern "C" {

const char* ttrl_last_error(void) { return g_last_error; }

int ttrl_version(void) { return 1; }

unsigned long long ttrl_launch_count(void) {
  return g_launches.load(std::memory_order_relaxed);
}

int ttrl_init(int device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return set_cuda_error("cudaSetDevice", e);
  const int rc = gemm_init_device();
  return rc != TTRL_OK ? rc : gru_init_device();
}

size_t ttrl_gemm_workspace_bytes(const ttrl_gemm_desc* d) {
  return d ? gemm_workspace_bytes(*d) : 0;
}

int ttrl_gemm(const ttrl_gemm_desc* d, float* workspace, size_t workspace_bytes, int* status,
              ttrl_stream_t stream) {
  if (d == nullptr) return set_error(TTRL_EINVAL, "ttrl_gemm: null descriptor");
  return gemm_run_ws(*d, 0, no_extra(), workspace, workspace_bytes, status, TTRL_STREAM(stream));
}

int ttrl_linear_fwd(const float* x, const float* w, const float* b, float* y, int m, int k, int n,
                    int relu, int precision, float* workspace, size_t workspace_bytes,
                    int* status, ttrl_stream_t stream) {
  return linear_fwd(x, w, b, y, m, k, n, relu, precision, workspace, workspace_bytes, status,
                    TTRL_STREAM(stream));
}

int ttrl_linear_dgrad(const float* g, const float* w, const float* mask, float* dx, int m, int k,
                      int n, int accumulate, int precision, float* workspace,
                      size_t workspace_bytes, int* status, ttrl_stream_t stream) {
  return linear_dgrad(g, w, mask, dx, m, k, n, accumulate, precision, workspace, workspace_bytes,
                      status, TTRL_STREAM(stream));
}

size_t ttrl_linear_wgrad_workspace_bytes(int m, int k, int n) {
  return (m > 0 && k > 0 && n > 0) ? linear_wgrad_ws(m, k, n) : 0;
}

int ttrl_linear_wgrad(const float* x, const float* g, float* dw, float* db, int m, int k, int n,
                      int accumulate, int accumulate_db, int precision, float* workspace,
                      size_t workspace_bytes, int* status, ttrl_stream_t stream) {
  return linear_wgrad(x, g, dw, db, m, k, n, accumulate, accumulate_db, precision, workspace,
                      workspace_bytes, status, TTRL_STREAM(stream));
}

int ttrl_conv_fprop(const float* x, const float* w, const float* b, float* y,
                    const ttrl_conv_geom* g, float alpha, int relu, int precision,
                    float* workspace, size_t workspace_bytes, int* status, ttrl_stream_t stream) {
  return conv_fprop(x, w, b, y, g, alpha, relu, precision, workspace, workspace_bytes, status,
                    TTRL_STREAM(stream));
}

int ttrl_conv_dgrad(const float* dy, const float* w, const float* mask, float* dx,
                    const ttrl_conv_geom* g, int accumulate, int precision, float* workspace,
                    size_t workspace_bytes, int* status, ttrl_stream_t stream) {
  return conv_dgrad(dy, w, mask, dx, g, accumulate, precision, workspace, workspace_bytes, status,
                    TTRL_STREAM(stream));
}

size_t ttrl_conv_dgrad_workspace_bytes(const ttrl_conv_geom* g) {
  return g ? conv_dgrad_ws(g) : 0;
}

size_t ttrl_conv_dgrad_weights_bytes(const ttrl_conv_geom* g) {
  return g ? conv_dgrad_weights_bytes(g) : 0;
}

int ttrl_conv_dgrad_weights(const float* w, float* out, const ttrl_conv_geom* g,
                            ttrl_stream_t stream) {
  return conv_dgrad_weights(w, out, g, TTRL_STREAM(stream));
}

int ttrl_conv_dgrad_prepared(const float* dy, const float* wt, const float* mask, float* dx,
                             const ttrl_conv_geom* g, int accumulate, int precision,
                             float* workspace, size_t workspace_bytes, int* status,
                             ttrl_stream_t stream) {
  return conv_dgrad_prepared(dy, wt, mask, dx, g, accumulate, precision, workspace,
                             workspace_bytes, status, TTRL_STREAM(stream));
}

size_t ttrl_conv_dgrad_prepared_workspace_bytes(const ttrl_conv_geom* g) {
  return g ? conv_dgrad_prepared_ws(g) : 0;
}

int ttrl_conv_wgrad(const float* x, const float* dy, float* dw, float* db,
                    const ttrl_conv_geom* g, float alpha, int accumulate, int accumulate_db,
                    int precision, float* workspace, size_t workspace_bytes, int* status,
                    ttrl_stream_t stream) {
  return conv_wgrad(x, dy, dw, db, g, alpha, accumulate, accumulate_db, precision, workspace,
                    workspace_bytes, status, TTRL_STREAM(stream));
}

size_t ttrl_conv_wgrad_workspace_bytes(const ttrl_conv_geom* g) {
  return g ? conv_wgrad_ws(g) : 0;
}

int ttrl_u8_nchw_to_f32_nhwc(const uint8_t* in, const int32_t* index, float* out, int n, int c,
                             int h, int w, float scale, ttrl_stream_t stream) {
  return u8_to_f32(in, index, out, n, c, h, w, scale, TTRL_STREAM(stream));
}

int ttrl_u8_nchw_to_f32_s2d(const uint8_t* in, const int32_t* index, float* out, int n, int c,
                            int h, int w, int fold, float scale, ttrl_stream_t stream) {
  return u8_to_f32_s2d(in, index, out, n, c, h, w, fold, scale, TTRL_STREAM(stream));
}

int ttrl_adam_step(const ttrl_adam_tensor* tensors, int count, int32_t* steps, int32_t* ticket,
                   const float* grad_scale, const double* lr_device, double lr, double b1,
                   double b2, double eps, double weight_decay, const double* bias_table,
                   int64_t bias_steps, ttrl_stream_t stream) {
  return adam_step(tensors, count, steps, ticket, grad_scale, lr_device, lr, b1, b2, eps,
                   weight_decay, bias_table, bias_steps, TTRL_STREAM(stream));
}

int ttrl_grad_sqnorm(const float* const* grads, const int64_t* numels, int count, float* out,
                     float max_norm, void* workspace, size_t workspace_bytes,
                     ttrl_stream_t stream) {
  return grad_sqnorm(grads, numels, count, out, max_norm, workspace, workspace_bytes,
                     TTRL_STREAM(stream));
}

size_t ttrl_grad_sqnorm_workspace_bytes(const int64_t* numels, int count) {
  return numels ? sqnorm_ws_bytes(numels, count) : 0;
}

int ttrl_ew(int op, const float* a, const int64_t* a_strides, const float* b,
            const int64_t* b_strides, float* out, const int64_t* shape, int ndim, float scalar,
            ttrl_stream_t stream) {
  return ew(op, a, a_strides, b, b_strides, out, shape, ndim, scalar, TTRL_STREAM(stream));
}

int ttrl_reduce(int op, const float* in, float* out, int64_t outer, int64_t n, int64_t inner,
                ttrl_stream_t stream) {
  return reduce(op, in, out, outer, n, inner, TTRL_STREAM(stream));
}

int ttrl_copy_strided(float* dst, const int64_t* dst_strides, const float* src,
                      const int64_t* src_strides, const int64_t* shape, int ndim, int accumulate,
                      ttrl_stream_t stream) {
  return copy_strided(dst, dst_strides, src, src_strides, shape, ndim, accumulate,
                      TTRL_STREAM(stream));
}

int ttrl_wait_probe(int* status, ttrl_stream_t stream) {
  return wait_probe(status, TTRL_STREAM(stream));
}

int ttrl_polyak(float* dst, const float* src, int64_t n, float tau, ttrl_stream_t stream) {
  return polyak(dst, src, n, tau, TTRL_STREAM(stream));
}

int ttrl_blend_multi(const ttrl_blend_pair* pairs, int count, int mode, float tau,
                     ttrl_stream_t stream) {
  return blend_multi(pairs, count, mode, tau, TTRL_STREAM(stream));
}

int ttrl_gather_rows(const void* src, const int32_t* idx, void* dst, int n, int row,
                     ttrl_stream_t stream) {
  return gather_rows(src, idx, dst, n, row, TTRL_STREAM(stream));
}

int ttrl_gather_rows_multi(const ttrl_gather_job* jobs, int count, const int32_t* idx, int n,
                           ttrl_stream_t stream) {
  return gather_rows_multi(jobs, count, idx, n, TTRL_STREAM(stream));
}

int ttrl_dqn_loss(const float* q, const float* q_sel, const float* q_tgt, const float* onehot,
                  const float* rewards, const float* dones, const float* discounts,
                  const float* next_mask, const float* is_weights, float* loss, float* mean_q,
                  float* td_abs, float* dq, int batch, int actions, float delta, int accumulate,
                  ttrl_stream_t stream) {
  DqnArgs a{q, q_sel, q_tgt, onehot, rewards, dones, discounts, next_mask, is_weights,
            loss, mean_q, td_abs, dq, batch, actions, delta, accumulate};
  return dqn_loss(a, TTRL_STREAM(stream));
}

int ttrl_ppo_loss(const float* logits, const float* value, const int32_t* actions,
                  const float* old_logp, const float* adv, const float* returns,
                  const float* old_values, const float* valid, float* metrics, float* new_logp,
                  float* dlogits, float* dvalue, int batch, int actions_n, float clip_eps,
                  float value_clip_eps, float value_coef, float entropy_coef,
                  ttrl_stream_t stream) {
  PpoArgs a{logits, value, actions, old_logp, adv, returns, old_values, valid, metrics,
            new_logp, dlogits, dvalue, batch, actions_n, clip_eps, value_clip_eps, value_coef,
            entropy_coef};
  return ppo_loss(a, TTRL_STREAM(stream));
}

}  // extern "C"
