// Flags in peer-mapped memory for the sharded parameter all-gather over
// NVLink copy engines. The owners' updated parameters move with
// cudaMemcpyAsync (copy engines, no SMs) while the Newton-Schulz kernels
// keep every SM; these two kernels order those copies across GPUs:
//   flags_set   one thread per flag: st.release.sys of `value` (the flag may
//               live in another GPU's memory, mapped into this one's address
//               space), after every write of the preceding kernels on the
//               stream;
//   flags_wait  one warp: lane i polls flag i with ld.acquire.sys until it
//               reaches `value` (wrap-around order), sleeping between polls;
//               the wait is bounded, and on expiry records kDevTimeoutFlag in
//               the device error word and returns.
// The reference gathers with torch.distributed collectives
// (opendm/optimizer/muon_adamw.py:503-535); this has no counterpart there.

#include "common.cuh"
#include "internal.h"

namespace muon {

__global__ void flags_set_kernel(muon_flag_list list, uint32_t value) {
  const int i = threadIdx.x;
  if (i < list.n) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(list.ptr[i]), "r"(value) : "memory");
  }
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void flags_wait_kernel(muon_flag_list list, uint32_t value, unsigned long long timeout_ns, int* err) {
  const int i = threadIdx.x;
  bool done = i >= list.n;
  const unsigned long long t0 = global_timer_ns();
  while (!done) {
    done = static_cast<int32_t>(ld_acquire_sys(list.ptr[i]) - value) >= 0;
    if (done) break;
    if (*reinterpret_cast<volatile int*>(err) != 0) break;  // another wait already failed
    if (global_timer_ns() - t0 > timeout_ns) {
      atomicCAS(err, 0, kDevTimeoutFlag);
      break;
    }
    __nanosleep(256);
  }
  __syncwarp();
}

int launch_flags_set(const muon_flag_list* list, uint32_t value, cudaStream_t stream) {
  if (!list) return set_error(MUON_ERR_ARG, "flag list is null");
  if (list->n < 0 || list->n > MUON_MAX_FLAGS) return set_error(MUON_ERR_ARG, "flag list size out of range");
  for (int i = 0; i < list->n; ++i)
    if (!list->ptr[i] || (reinterpret_cast<uintptr_t>(list->ptr[i]) & 3u) != 0)
      return set_error(MUON_ERR_ARG, "flag pointer is null or not 4-byte aligned");
  if (list->n == 0) return MUON_OK;
  flags_set_kernel<<<1, 32, 0, stream>>>(*list, value);
  return check_cuda(cudaGetLastError(), "flags_set launch");
}

int launch_flags_wait(const muon_flag_list* list, uint32_t value, int64_t timeout_us, int* err_dev,
                      cudaStream_t stream) {
  if (!list || !err_dev) return set_error(MUON_ERR_ARG, "flag list or error word is null");
  if (list->n < 0 || list->n > MUON_MAX_FLAGS) return set_error(MUON_ERR_ARG, "flag list size out of range");
  if (timeout_us <= 0) return set_error(MUON_ERR_ARG, "timeout_us must be positive");
  for (int i = 0; i < list->n; ++i)
    if (!list->ptr[i] || (reinterpret_cast<uintptr_t>(list->ptr[i]) & 3u) != 0)
      return set_error(MUON_ERR_ARG, "flag pointer is null or not 4-byte aligned");
  if (list->n == 0) return MUON_OK;
  flags_wait_kernel<<<1, 32, 0, stream>>>(*list, value, static_cast<unsigned long long>(timeout_us) * 1000ull,
                                          err_dev);
  return check_cuda(cudaGetLastError(), "flags_wait launch");
}

}  // namespace muon
