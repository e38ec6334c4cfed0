// Internal (C++) interface between the C-ABI layer and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "opendm_muon.h"

namespace muon {

// Records a failure for muon_last_error() and returns `code`.
int set_error(int code, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);

int launch_momentum(const muon_momentum_seg* segs_dev, int n_segs, int64_t total_chunks,
                    int grad_dtype, int dir_dtype, float momentum, int nesterov, float eps,
                    float* partials_dev, float* scales_dev, const float* grad_scale, cudaStream_t stream);
int64_t momentum_chunks(int64_t rows, int64_t cols);
int launch_momentum_single_noalloc(const void* grad, float* exp_avg, void* direction, int64_t rows, int64_t cols,
                                   int64_t ld, int grad_dtype, int dir_dtype, float momentum, int nesterov,
                                   float eps, float* scale_out, cudaStream_t stream);

int launch_adamw(const muon_adamw_seg* segs_dev, int n_segs, int64_t total_chunks, double beta1,
                 double beta2, float eps, float wd_factor, const float* grad_scale, cudaStream_t stream);
int64_t norm_chunks(int64_t numel);
int launch_clip_grad_norm(const muon_norm_seg* segs_dev, int n_segs, int64_t total_chunks, float max_norm,
                          float* partials_dev, float* out_dev, cudaStream_t stream);
int64_t adamw_chunks(int64_t numel);

int ns_plan_create(const muon_ns_class* classes, int n_classes, int op_dtype, int steps,
                   muon_ns_plan** plan_out);
int ns_plan_run(const muon_ns_plan* plan, int* err_dev, cudaStream_t stream);
int launch_apply_update(const muon_update_seg* segs_dev, int n_segs, int64_t total_chunks, float wd_factor,
                        cudaStream_t stream);
void ns_plan_destroy(muon_ns_plan* plan);
int ns_plan_launches(const muon_ns_plan* plan);
int ns_plan_set_sm_limit(muon_ns_plan* plan, int sms);
int64_t ns_class_workspace_bytes(int32_t rows, int32_t cols, int32_t count, int op_dtype, int algo);
int ns_choose_algo(int32_t rows, int32_t cols, int op_dtype, int steps);
int ns_gram_segment(int op_dtype);
int ns_class_layout(muon_ns_class* cls, void* base, int op_dtype);
float ns_operand_scale(int32_t rows, int32_t cols, int iteration, int op_dtype);

int launch_flags_set(const muon_flag_list* list, uint32_t value, cudaStream_t stream);
int launch_flags_wait(const muon_flag_list* list, uint32_t value, int64_t timeout_us, int* err_dev,
                      cudaStream_t stream);

int launch_momentum_f16(const muon_momentum_f16_seg* segs_dev, int n_segs, int64_t total_chunks, int grad_dtype,
                        float momentum, int nesterov, float eps, float* partials_dev, float* pscale_dev,
                        float* scales_dev, int* redo_dev, const float* grad_scale, cudaStream_t stream);
}  // namespace muon
