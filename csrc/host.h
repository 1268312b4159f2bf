// Host-side helpers shared by the revpp CUDA extension.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>

// Argument checks throw std::runtime_error (pybind11 maps it to RuntimeError).
// c10::Error thrown through host code built by g++ here crashed the process
// instead of reaching Python, so the extension never uses TORCH_CHECK.
#define REVPP_CHECK(cond, ...)                                                              \
  do {                                                                                      \
    if (!(cond)) {                                                                          \
      throw std::runtime_error(c10::str("revpp: check failed [", #cond, "] at ", __FILE__, ":", \
                                        __LINE__, " ", ##__VA_ARGS__));                     \
    }                                                                                       \
  } while (0)

#define REVPP_CUDA_CHECK(expr)                                                                      \
  do {                                                                                              \
    cudaError_t _e = (expr);                                                                        \
    REVPP_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " (", #expr, ")");         \
  } while (0)

#define REVPP_CHECK_LAUNCH()               \
  do {                                     \
    REVPP_CUDA_CHECK(cudaGetLastError());  \
    ::revpp::count_launch();               \
  } while (0)

namespace revpp {

// Number of kernels this process has launched through the extension.
void count_launch();
int64_t launch_count();

// Device pointer of this process's status word for the current device.  Kernels
// OR error bits into it; the host reads it through the mapped pinned page
// without a device synchronisation.
int* status_device_ptr();
int status_peek();
int status_read_and_clear();

int num_sms();
// SMs a persistent kernel may fill: all SMs minus those left free for concurrent
// communication kernels (set_sm_reserve).
int gemm_grid_sms();
void set_sm_reserve(int n);
int sm_reserve();
int max_smem_optin();

// 2-D bf16 tensor map for TMA.  inner = elements of the contiguous dimension,
// outer = number of rows, row_stride_bytes must be a multiple of 16.
CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                         uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle);

inline void check_cuda_bf16(const torch::Tensor& t, const char* name) {
  REVPP_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  REVPP_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
}
inline void check_cuda_f32(const torch::Tensor& t, const char* name) {
  REVPP_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  REVPP_CHECK(t.scalar_type() == at::kFloat, name, " must be float32");
}

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Programmatic dependent launch (on unless REVPP_PDL=0): kernels of this extension that
// call pdl_wait() before touching memory written by earlier work of the stream (and
// pdl_trigger() right after) are launched with the programmatic-serialization attribute,
// so each one's launch and set-up (barriers, TMEM, descriptor prefetch) overlap the tail of
// the kernel before it.  An operation other than a kernel in between (an event wait, a
// copy) keeps the ordinary dependency.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  REVPP_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

}  // namespace revpp
