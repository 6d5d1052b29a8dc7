// extern "C" boundary of libddpm_b200.so: argument checks, thread-local error
// text, and forwarding into the kernel launchers. Declarations and the
// reference interface each entry point replaces are in include/ddpm_b200.h.
#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace ddpm {

namespace {
thread_local char g_last_error[512] = "";
std::atomic<unsigned long long> g_launches{0};
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = '\0'; }

int dyncat_fwd(const void* x, int xdt, const void* k, int kdt, void* out, int n, int c, int h,
               int w, int ks, int d0, int d1, int d2, cudaStream_t st);
int dyncat_bwd(const void* x, int xdt, const void* k, const void* g, int kdt, void* gx, void* gk,
               int n, int c, int h, int w, int ks, int d0, int d1, int d2, cudaStream_t st);

int gencat_fwd_test_skip_arrive(int enable);
int dyncat_set_tma_disabled(int disabled);
int umma_selftest(int variant, const void* a, const void* b, float* d, int n, int k, int shift,
                  cudaStream_t st);

size_t gencat_pack_bytes(int c, int ks, int dt);
int gencat_pack(const void* w, const void* bias, int c, int ks, int dt, void* packed,
                size_t packed_bytes, cudaStream_t st);
int gencat_fwd(const void* x, const void* y, const void* staged, size_t staged_bytes,
               const void* wpack, const void* bias, void* out, int n, int c, int h, int w,
               int ks, int d0, int d1, int d2, int dt, cudaStream_t st);
int gencat_fwd_ex(const void* x, const void* y, const void* staged, size_t staged_bytes,
                  const void* wpack, const void* bias, void* out, void* planes,
                  size_t planes_bytes, int n, int c, int h, int w, int ks, int d0, int d1,
                  int d2, int dt, cudaStream_t st);

int gencat_bwd_x(const void* y, const void* staged, size_t staged_bytes, const void* wpack,
                 const void* bias, const void* gout, void* gx, int n, int c, int h, int w, int ks,
                 int d0, int d1, int d2, int dt, cudaStream_t st, int g_nhwc);
namespace gencat {
size_t stage_bytes(int n, int c, int h, int w, int ks, int d0, int d1, int d2, int dt);
int stage(const void* x, const void* y, void* staged, size_t staged_bytes, int n, int c, int h,
          int w, int ks, int d0, int d1, int d2, int dt, cudaStream_t st);
}  // namespace gencat

size_t gencat_bwd_workspace_bytes(int n, int c, int h, int w, int ks);
int gencat_bwd_yw(const void* x, const void* y, const void* staged, size_t staged_bytes,
                  const void* wpack, const void* gout, void* gy, void* gw, void* gb,
                  void* workspace, size_t ws_bytes, int n, int c, int h, int w, int ks, int d0,
                  int d1, int d2, int dt, cudaStream_t st, int g_nhwc);

int gencat_bwd_yw_static(const void* x, const void* y, const void* wpack, const void* gout,
                         void* gy, void* gw, void* gb, int n, int c, int h, int w, int ks, int d0,
                         int d1, int d2, int dt, cudaStream_t st);
size_t fuseconv_pack_bytes(int cin, int cout, int dt);
int fuseconv_pack(const void* w, int cin, int cout, int dt, void* packed, size_t bytes,
                  cudaStream_t st);
int fuseconv_fwd(const void* cat, const void* packed, const void* bias, void* out, int n, int cin,
                 int cout, int h, int w, int dt, cudaStream_t st);
int fuseconv_dgrad(const void* gout, const void* packed, void* gcat, int n, int cin, int cout,
                   int h, int w, int dt, cudaStream_t st, int gcat_nhwc);
int fuseconv_bwd(const void* cat, const void* gout, const void* packed, void* gcat, void* gw,
                 void* gb, void* ws, size_t ws_bytes, int n, int cin, int cout, int h, int w,
                 int dt, cudaStream_t st, int gcat_nhwc);
size_t fuseconv_stage_bytes(int n, int c, int h, int w, int dt);
int fuseconv_stage(const void* src, void* planes, size_t bytes, int n, int c, int h, int w, int dt,
                   cudaStream_t st);
int fuseconv_fwd_staged(const void* planes, size_t planes_bytes, const void* packed,
                        const void* bias, void* out, int n, int cin, int cout, int h, int w, int dt,
                        cudaStream_t st);
int fuseconv_dgrad_staged(const void* planes, size_t planes_bytes, const void* packed, void* gcat,
                          int n, int cin, int cout, int h, int w, int dt, cudaStream_t st);
namespace gencat {
int read_status(int reset, int* code);
}
size_t fuseconv_wgrad_workspace_bytes(int n, int cin, int cout, int h, int w);
int fuseconv_wgrad(const void* cat, const void* gout, void* gw, void* gb, void* ws, size_t ws_bytes,
                   int n, int cin, int cout, int h, int w, int dt, cudaStream_t st);
}  // namespace ddpm

extern "C" {

int ddpm_version(void) { return 100; }

const char* ddpm_last_error(void) { return ddpm::g_last_error; }

unsigned long long ddpm_launch_count(void) {
  return ddpm::g_launches.load(std::memory_order_relaxed);
}

int ddpm_dyncat_fwd(const void* x, int x_dtype, const void* kernels, int k_dtype, void* out, int n,
                    int c, int h, int w, int ksize, int d0, int d1, int d2, void* stream) {
  ddpm::clear_error();
  return ddpm::dyncat_fwd(x, x_dtype, kernels, k_dtype, out, n, c, h, w, ksize, d0, d1, d2,
                          static_cast<cudaStream_t>(stream));
}

int ddpm_dyncat_bwd(const void* x, int x_dtype, const void* kernels, const void* grad_out,
                    int k_dtype, void* grad_x, void* grad_k, int n, int c, int h, int w, int ksize,
                    int d0, int d1, int d2, void* stream) {
  ddpm::clear_error();
  return ddpm::dyncat_bwd(x, x_dtype, kernels, grad_out, k_dtype, grad_x, grad_k, n, c, h, w,
                          ksize, d0, d1, d2, static_cast<cudaStream_t>(stream));
}

int ddpm_test_disable_tma(int disabled) {
  ddpm::clear_error();
  return ddpm::dyncat_set_tma_disabled(disabled);
}

int ddpm_test_skip_arrive(int enable) {
  ddpm::clear_error();
  return ddpm::gencat_fwd_test_skip_arrive(enable);
}

int ddpm_umma_selftest(int variant, const void* a, const void* b, float* d, int n, int k,
                       int shift, void* stream) {
  ddpm::clear_error();
  return ddpm::umma_selftest(variant, a, b, d, n, k, shift, static_cast<cudaStream_t>(stream));
}

size_t ddpm_gencat_pack_bytes(int c, int ksize, int dtype) {
  return ddpm::gencat_pack_bytes(c, ksize, dtype);
}

int ddpm_gencat_pack(const void* weight, const void* bias, int c, int ksize, int dtype,
                     void* packed, size_t packed_bytes, void* stream) {
  ddpm::clear_error();
  return ddpm::gencat_pack(weight, bias, c, ksize, dtype, packed, packed_bytes,
                           static_cast<cudaStream_t>(stream));
}

int ddpm_gencat_fwd(const void* x, const void* y, const void* packed, const void* bias, void* out,
                    int n, int c, int h, int w, int ksize, int d0, int d1, int d2, int dtype,
                    void* stream) {
  ddpm::clear_error();
  return ddpm::gencat_fwd(x, y, nullptr, 0, packed, bias, out, n, c, h, w, ksize, d0, d1, d2,
                          dtype, static_cast<cudaStream_t>(stream));
}

int ddpm_gencat_fwd_staged_planes(const void* staged, size_t staged_bytes, const void* packed,
                                  const void* bias, void* out, void* planes, size_t planes_bytes,
                                  int n, int c, int h, int w, int ksize, int d0, int d1, int d2,
                                  int dtype, void* stream) {
  ddpm::clear_error();
  DDPM_CHECK_ARG(staged && planes, "null pointer");
  return ddpm::gencat_fwd_ex(nullptr, nullptr, staged, staged_bytes, packed, bias, out, planes,
                             planes_bytes, n, c, h, w, ksize, d0, d1, d2, dtype,
                             static_cast<cudaStream_t>(stream));
}

int ddpm_gencat_fwd_staged(const void* staged, size_t staged_bytes, const void* packed,
                           const void* bias, void* out, int n, int c, int h, int w, int ksize,
                           int d0, int d1, int d2, int dtype, void* stream) {
  ddpm::clear_error();
  DDPM_CHECK_ARG(staged != nullptr, "null staged");
  return ddpm::gencat_fwd(nullptr, nullptr, staged, staged_bytes, packed, bias, out, n, c, h, w,
                          ksize, d0, d1, d2, dtype, static_cast<cudaStream_t>(stream));
}

int ddpm_gencat_bwd_x(const void* y, const void* packed, const void* bias, const void* grad_out,
                      void* grad_x, int n, int c, int h, int w, int ksize, int d0, int d1, int d2,
                      int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::gencat_bwd_x(y, nullptr, 0, packed, bias, grad_out, grad_x, n, c, h, w, ksize, d0,
                            d1, d2, dtype, static_cast<cudaStream_t>(stream), 0);
}

size_t ddpm_gencat_stage_bytes(int n, int c, int h, int w, int ksize, int d0, int d1, int d2,
                               int dtype) {
  return ddpm::gencat::stage_bytes(n, c, h, w, ksize, d0, d1, d2, dtype);
}

int ddpm_gencat_stage(const void* x, const void* y, void* staged, size_t staged_bytes, int n,
                      int c, int h, int w, int ksize, int d0, int d1, int d2, int dtype,
                      void* stream) {
  ddpm::clear_error();
  return ddpm::gencat::stage(x, y, staged, staged_bytes, n, c, h, w, ksize, d0, d1, d2, dtype,
                             static_cast<cudaStream_t>(stream));
}

int ddpm_gencat_bwd_x_staged(const void* staged_y, size_t staged_bytes, const void* packed,
                             const void* bias, const void* grad_out, void* grad_x, int n, int c,
                             int h, int w, int ksize, int d0, int d1, int d2, int dtype,
                             void* stream) {
  ddpm::clear_error();
  DDPM_CHECK_ARG(staged_y != nullptr, "null staged_y");
  return ddpm::gencat_bwd_x(nullptr, staged_y, staged_bytes, packed, bias, grad_out, grad_x, n, c,
                            h, w, ksize, d0, d1, d2, dtype, static_cast<cudaStream_t>(stream), 0);
}

int ddpm_gencat_bwd_x_staged_nhwc(const void* staged_y, size_t staged_bytes, const void* packed,
                                  const void* bias, const void* grad_out, void* grad_x, int n,
                                  int c, int h, int w, int ksize, int d0, int d1, int d2,
                                  int dtype, void* stream) {
  ddpm::clear_error();
  DDPM_CHECK_ARG(staged_y != nullptr, "null staged_y");
  return ddpm::gencat_bwd_x(nullptr, staged_y, staged_bytes, packed, bias, grad_out, grad_x, n, c,
                            h, w, ksize, d0, d1, d2, dtype, static_cast<cudaStream_t>(stream), 1);
}

size_t ddpm_gencat_bwd_workspace_bytes(int n, int c, int h, int w, int ksize) {
  return ddpm::gencat_bwd_workspace_bytes(n, c, h, w, ksize);
}

int ddpm_gencat_bwd_yw(const void* x, const void* y, const void* packed, const void* grad_out,
                       void* grad_y, void* grad_weight, void* grad_bias, void* workspace,
                       size_t workspace_bytes, int n, int c, int h, int w, int ksize, int d0,
                       int d1, int d2, int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::gencat_bwd_yw(x, y, nullptr, 0, packed, grad_out, grad_y, grad_weight, grad_bias,
                             workspace, workspace_bytes, n, c, h, w, ksize, d0, d1, d2, dtype,
                             static_cast<cudaStream_t>(stream), 0);
}

int ddpm_gencat_bwd_yw_staged(const void* staged, size_t staged_bytes, const void* packed,
                              const void* grad_out, void* grad_y, void* grad_weight,
                              void* grad_bias, void* workspace, size_t ws_bytes, int n, int c,
                              int h, int w, int ksize, int d0, int d1, int d2, int dtype,
                              void* stream) {
  ddpm::clear_error();
  DDPM_CHECK_ARG(staged != nullptr, "null staged");
  return ddpm::gencat_bwd_yw(nullptr, nullptr, staged, staged_bytes, packed, grad_out, grad_y,
                             grad_weight, grad_bias, workspace, ws_bytes, n, c, h, w, ksize, d0,
                             d1, d2, dtype, static_cast<cudaStream_t>(stream), 0);
}

int ddpm_gencat_bwd_yw_staged_nhwc(const void* staged, size_t staged_bytes, const void* packed,
                                   const void* grad_out, void* grad_y, void* grad_weight,
                                   void* grad_bias, void* workspace, size_t ws_bytes, int n,
                                   int c, int h, int w, int ksize, int d0, int d1, int d2,
                                   int dtype, void* stream) {
  ddpm::clear_error();
  DDPM_CHECK_ARG(staged != nullptr, "null staged");
  return ddpm::gencat_bwd_yw(nullptr, nullptr, staged, staged_bytes, packed, grad_out, grad_y,
                             grad_weight, grad_bias, workspace, ws_bytes, n, c, h, w, ksize, d0,
                             d1, d2, dtype, static_cast<cudaStream_t>(stream), 1);
}

int ddpm_gencat_bwd_yw_static(const void* x, const void* y, const void* packed,
                              const void* grad_out, void* grad_y, void* grad_weight,
                              void* grad_bias, int n, int c, int h, int w, int ksize, int d0,
                              int d1, int d2, int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::gencat_bwd_yw_static(x, y, packed, grad_out, grad_y, grad_weight, grad_bias, n, c,
                                    h, w, ksize, d0, d1, d2, dtype,
                                    static_cast<cudaStream_t>(stream));
}

size_t ddpm_fuseconv_pack_bytes(int cin, int cout, int dtype) {
  return ddpm::fuseconv_pack_bytes(cin, cout, dtype);
}

int ddpm_fuseconv_pack(const void* weight, int cin, int cout, int dtype, void* packed,
                       size_t packed_bytes, void* stream) {
  ddpm::clear_error();
  return ddpm::fuseconv_pack(weight, cin, cout, dtype, packed, packed_bytes,
                             static_cast<cudaStream_t>(stream));
}

int ddpm_fuseconv_fwd(const void* x, const void* packed, const void* bias, void* out, int n,
                      int cin, int cout, int h, int w, int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::fuseconv_fwd(x, packed, bias, out, n, cin, cout, h, w, dtype,
                            static_cast<cudaStream_t>(stream));
}

int ddpm_fuseconv_bwd_data(const void* grad_out, const void* packed, void* grad_x, int n,
                           int cin, int cout, int h, int w, int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::fuseconv_dgrad(grad_out, packed, grad_x, n, cin, cout, h, w, dtype,
                              static_cast<cudaStream_t>(stream), 0);
}

int ddpm_fuseconv_bwd(const void* x, const void* grad_out, const void* packed, void* grad_x,
                      void* grad_weight, void* grad_bias, void* workspace, size_t workspace_bytes,
                      int n, int cin, int cout, int h, int w, int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::fuseconv_bwd(x, grad_out, packed, grad_x, grad_weight, grad_bias, workspace,
                            workspace_bytes, n, cin, cout, h, w, dtype,
                            static_cast<cudaStream_t>(stream), 0);
}

int ddpm_fuseconv_bwd_nhwc(const void* x, const void* grad_out, const void* packed, void* grad_x,
                           void* grad_weight, void* grad_bias, void* workspace,
                           size_t workspace_bytes, int n, int cin, int cout, int h, int w,
                           int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::fuseconv_bwd(x, grad_out, packed, grad_x, grad_weight, grad_bias, workspace,
                            workspace_bytes, n, cin, cout, h, w, dtype,
                            static_cast<cudaStream_t>(stream), 1);
}

size_t ddpm_fuseconv_stage_bytes(int n, int c, int h, int w, int dtype) {
  return ddpm::fuseconv_stage_bytes(n, c, h, w, dtype);
}

int ddpm_fuseconv_stage(const void* src, void* planes, size_t planes_bytes, int n, int c, int h,
                        int w, int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::fuseconv_stage(src, planes, planes_bytes, n, c, h, w, dtype,
                              static_cast<cudaStream_t>(stream));
}

int ddpm_fuseconv_fwd_staged(const void* planes, size_t planes_bytes, const void* packed,
                             const void* bias, void* out, int n, int cin, int cout, int h, int w,
                             int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::fuseconv_fwd_staged(planes, planes_bytes, packed, bias, out, n, cin, cout, h, w,
                                   dtype, static_cast<cudaStream_t>(stream));
}

int ddpm_fuseconv_bwd_data_staged(const void* planes, size_t planes_bytes, const void* packed,
                                  void* grad_x, int n, int cin, int cout, int h, int w, int dtype,
                                  void* stream) {
  ddpm::clear_error();
  return ddpm::fuseconv_dgrad_staged(planes, planes_bytes, packed, grad_x, n, cin, cout, h, w,
                                     dtype, static_cast<cudaStream_t>(stream));
}

int ddpm_device_status(int reset, int* code) {
  ddpm::clear_error();
  return ddpm::gencat::read_status(reset, code);
}

size_t ddpm_fuseconv_bwd_weight_workspace_bytes(int n, int cin, int cout, int h, int w) {
  return ddpm::fuseconv_wgrad_workspace_bytes(n, cin, cout, h, w);
}

int ddpm_fuseconv_bwd_weight(const void* x, const void* grad_out, void* grad_weight,
                             void* grad_bias, void* workspace, size_t workspace_bytes, int n,
                             int cin, int cout, int h, int w, int dtype, void* stream) {
  ddpm::clear_error();
  return ddpm::fuseconv_wgrad(x, grad_out, grad_weight, grad_bias, workspace, workspace_bytes, n,
                              cin, cout, h, w, dtype, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
