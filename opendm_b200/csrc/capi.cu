// extern "C" entry points declared in include/opendm_muon.h. Each forwards to
// the kernel file that implements it; this file owns error reporting.

#include <cstdio>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace muon {

// Waits on an mbarrier phase that nothing completes, with a caller-chosen
// bound: exercises the timeout path of every pipeline wait in this library.
__global__ void selftest_wait_kernel(int* err, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, err, kDevSelftest, timeout_ns);
}

static thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MUON_OK;
  char buf[256];
  snprintf(buf, sizeof(buf), "%s: %s (%d)", what, cudaGetErrorString(e), int(e));
  return set_error(MUON_ERR_CUDA, buf);
}

}  // namespace muon

using muon::set_error;

extern "C" {

int muon_version(void) { return MUON_ABI_VERSION; }

const char* muon_last_error(void) { return muon::g_last_error.c_str(); }

int muon_device_check(int device) {
  int major = 0, minor = 0;
  if (muon::check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device),
                       "compute capability"))
    return MUON_ERR_CUDA;
  if (muon::check_cuda(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device),
                       "compute capability"))
    return MUON_ERR_CUDA;
  if (major != 10 || minor != 0) {
    char buf[128];
    snprintf(buf, sizeof(buf), "device %d is sm_%d%d; this library is built for sm_100a only", device,
             major, minor);
    return set_error(MUON_ERR_DEVICE, buf);
  }
  return MUON_OK;
}

int muon_read_error(int* err_dev, int* host_code, void* stream) {
  if (!err_dev || !host_code) return set_error(MUON_ERR_ARG, "null error pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int code = 0;
  if (muon::check_cuda(cudaMemcpyAsync(&code, err_dev, sizeof(int), cudaMemcpyDeviceToHost, s),
                       "read error word"))
    return MUON_ERR_CUDA;
  if (muon::check_cuda(cudaStreamSynchronize(s), "stream synchronize")) return MUON_ERR_CUDA;
  *host_code = code;
  if (code != 0) {
    if (muon::check_cuda(cudaMemsetAsync(err_dev, 0, sizeof(int), s), "clear error word"))
      return MUON_ERR_CUDA;
    char buf[128];
    snprintf(buf, sizeof(buf), "kernel reported error code 0x%x (bounded wait expired)", code);
    return set_error(MUON_ERR_KERNEL, buf);
  }
  return MUON_OK;
}

int muon_selftest_bounded_wait(int* err_dev, int timeout_us, void* stream) {
  if (!err_dev) return set_error(MUON_ERR_ARG, "err_dev is null");
  if (timeout_us < 1 || timeout_us > 1000000) return set_error(MUON_ERR_ARG, "timeout_us must be in [1, 1e6]");
  muon::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      err_dev, 1000ull * static_cast<unsigned long long>(timeout_us));
  return muon::check_cuda(cudaGetLastError(), "selftest launch");
}

int64_t muon_momentum_chunks(int64_t rows, int64_t cols) { return muon::momentum_chunks(rows, cols); }

int muon_momentum(const muon_momentum_seg* segs_dev, int n_segs, int64_t total_chunks, int grad_dtype,
                  int dir_dtype, float momentum, int nesterov, float eps, float* partials_dev,
                  float* scales_dev, void* stream) {
  return muon::launch_momentum(segs_dev, n_segs, total_chunks, grad_dtype, dir_dtype, momentum, nesterov,
                               eps, partials_dev, scales_dev, nullptr, static_cast<cudaStream_t>(stream));
}

int muon_momentum_scaled(const muon_momentum_seg* segs_dev, int n_segs, int64_t total_chunks, int grad_dtype,
                         int dir_dtype, float momentum, int nesterov, float eps, float* partials_dev,
                         float* scales_dev, const float* grad_scale_dev, void* stream) {
  return muon::launch_momentum(segs_dev, n_segs, total_chunks, grad_dtype, dir_dtype, momentum, nesterov,
                               eps, partials_dev, scales_dev, grad_scale_dev, static_cast<cudaStream_t>(stream));
}

int muon_momentum_single_noalloc(const void* grad, float* exp_avg, void* direction, int64_t rows, int64_t cols,
                                 int64_t ld, int grad_dtype, int dir_dtype, float momentum, int nesterov, float eps,
                                 float* scale_out, void* stream) {
  return muon::launch_momentum_single_noalloc(grad, exp_avg, direction, rows, cols, ld, grad_dtype, dir_dtype,
                                              momentum, nesterov, eps, scale_out, static_cast<cudaStream_t>(stream));
}

float muon_ns_operand_scale(int32_t rows, int32_t cols, int iteration, int op_dtype) {
  return muon::ns_operand_scale(rows, cols, iteration, op_dtype);
}

int muon_ns_plan_create(const muon_ns_class* classes, int n_classes, int op_dtype, int steps,
                        muon_ns_plan** plan_out) {
  if (!classes) return set_error(MUON_ERR_ARG, "classes is null");
  return muon::ns_plan_create(classes, n_classes, op_dtype, steps, plan_out);
}

int muon_ns_plan_run(const muon_ns_plan* plan, int* err_dev, void* stream) {
  return muon::ns_plan_run(plan, err_dev, static_cast<cudaStream_t>(stream));
}

int muon_apply_update(const muon_update_seg* segs_dev, int n_segs, int64_t total_chunks, float wd_factor,
                      void* stream) {
  return muon::launch_apply_update(segs_dev, n_segs, total_chunks, wd_factor, static_cast<cudaStream_t>(stream));
}

void muon_ns_plan_destroy(muon_ns_plan* plan) { muon::ns_plan_destroy(plan); }

int muon_ns_plan_launches(const muon_ns_plan* plan) { return muon::ns_plan_launches(plan); }

int muon_flags_set(const muon_flag_list* list, uint32_t value, void* stream) {
  return muon::launch_flags_set(list, value, static_cast<cudaStream_t>(stream));
}

int muon_flags_wait(const muon_flag_list* list, uint32_t value, int64_t timeout_us, int* err_dev, void* stream) {
  return muon::launch_flags_wait(list, value, timeout_us, err_dev, static_cast<cudaStream_t>(stream));
}

int muon_ns_plan_set_sm_limit(muon_ns_plan* plan, int sms) { return muon::ns_plan_set_sm_limit(plan, sms); }

int64_t muon_ns_class_workspace_bytes(int32_t rows, int32_t cols, int32_t count, int op_dtype, int algo) {
  return muon::ns_class_workspace_bytes(rows, cols, count, op_dtype, algo);
}

int muon_ns_choose_algo(int32_t rows, int32_t cols, int op_dtype, int steps) {
  return muon::ns_choose_algo(rows, cols, op_dtype, steps);
}

int muon_ns_gram_segment(int op_dtype) { return muon::ns_gram_segment(op_dtype); }

int muon_ns_class_layout(muon_ns_class* cls, void* base, int op_dtype) {
  return muon::ns_class_layout(cls, base, op_dtype);
}

int64_t muon_adamw_chunks(int64_t numel) { return muon::adamw_chunks(numel); }

int muon_adamw(const muon_adamw_seg* segs_dev, int n_segs, int64_t total_chunks, double beta1, double beta2,
               float eps, float wd_factor, void* stream) {
  return muon::launch_adamw(segs_dev, n_segs, total_chunks, beta1, beta2, eps, wd_factor, nullptr,
                            static_cast<cudaStream_t>(stream));
}

int muon_adamw_scaled(const muon_adamw_seg* segs_dev, int n_segs, int64_t total_chunks, double beta1, double beta2,
                      float eps, float wd_factor, const float* grad_scale_dev, void* stream) {
  return muon::launch_adamw(segs_dev, n_segs, total_chunks, beta1, beta2, eps, wd_factor, grad_scale_dev,
                            static_cast<cudaStream_t>(stream));
}

int64_t muon_norm_chunks(int64_t numel) { return muon::norm_chunks(numel); }

int muon_momentum_f16(const muon_momentum_f16_seg* segs_dev, int n_segs, int64_t total_chunks, int grad_dtype,
                      float momentum, int nesterov, float eps, float* partials_dev, float* pscale_dev,
                      float* scales_dev, int* redo_dev, const float* grad_scale_dev, void* stream) {
  return muon::launch_momentum_f16(segs_dev, n_segs, total_chunks, grad_dtype, momentum, nesterov, eps, partials_dev,
                                   pscale_dev, scales_dev, redo_dev, grad_scale_dev,
                                   static_cast<cudaStream_t>(stream));
}

int muon_clip_grad_norm(const muon_norm_seg* segs_dev, int n_segs, int64_t total_chunks, float max_norm,
                        float* partials_dev, float* out_dev, void* stream) {
  return muon::launch_clip_grad_norm(segs_dev, n_segs, total_chunks, max_norm, partials_dev, out_dev,
                                     static_cast<cudaStream_t>(stream));
}

}  // extern "C"
