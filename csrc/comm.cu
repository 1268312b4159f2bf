// Cross-GPU kernels over NVLink peer memory, and the bounded-wait primitives they use.
//
// dp_reduce_adamw: gradient all-reduce across D pipeline replicas fused with the gradient
// average, the clip-norm and the AdamW update, in one cooperative kernel per GPU.  Every
// rank maps its peers' flat buffers (CUDA IPC) and
//   0. flag barrier: every replica's backward has finished writing its gradients;
//   A. reduces its own shard r: g = (sum_d grad_d[shard r]) / D, read from the peers with
//      plain loads over NVLink, written back into its own grad[shard r]; squared-norm
//      partials accumulate on the way;
//   B. publishes its partial squared norm into every peer's flag page and raises its epoch
//      flag there (system-scope fence first); waits, with a time limit, until every peer's
//      flag in its own page shows this epoch, and sums the norms: clip coefficient;
//   C. applies AdamW to shard r (own m / v) and stores the new fp32 parameters and the bf16
//      shadow into its own buffers *and every peer's*; zeroes its whole gradient buffer
//      (the peers finished reading it before step B's barrier);
//   D. second flag barrier: no rank leaves until every peer's parameter stores are visible.
// Traffic per rank: (D-1)/D of the gradient in, (D-1)/D of the parameters (fp32 + bf16)
// out, no intermediate copies.  No TMA is used here, so no multicast load can touch peer
// memory.  Every wait gives up after `timeout_ns`, records kStatusFlagTimeout, writes an
// abort mark into every replica's flag page (so peers still waiting, or about to start
// step C, skip the update instead of leaving the replicas with mixed old and new shards)
// and returns; the trainer raises on the status bit at the end of the step.
//
// flag_wait_probe: a one-thread kernel that waits on a flag nobody sets, used by tests to
// check that the bounded wait reports an error instead of hanging.
#include <cooperative_groups.h>

#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "host.h"

namespace cg = cooperative_groups;

namespace revpp {

constexpr int kMaxPeers = 8;
// flag page layout (int32 words): [0, 64) epoch flags per rank, [64, 72) norm bits per rank,
// word 127 the abort mark (the epoch base of the next call, written by a rank that gave up)
constexpr int kFlagEpoch = 0;
constexpr int kFlagNorm = 64;
constexpr int kFlagAbort = 127;
constexpr int kFlagWords = 128;

struct DpArgs {
  float* grad[kMaxPeers];
  float* param[kMaxPeers];
  __nv_bfloat16* shadow[kMaxPeers];
  int* flags[kMaxPeers];
  float* m;
  float* v;
  float* sumsq_scratch;  // own, 2 floats
  long long n;           // elements in the flat buffers (multiple of 4 * D)
  int D, rank, epoch, zero_grad;
  float lr, beta1, beta2, eps, wd, step_size, inv_bc2_sqrt, max_norm, inv_d;
  long long timeout_ns;
  int* status;
};

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
__device__ __forceinline__ void st_volatile(int* p, int v) { *reinterpret_cast<volatile int*>(p) = v; }

// True once some rank has marked this call (epoch base `base`) as aborted in our page.
__device__ __forceinline__ bool aborted(const int* own_flags, int base) {
  return ld_volatile(own_flags + kFlagAbort) > base;
}

// Mark the call aborted in every replica's page (best effort: a peer that is already past
// its last check completes the update, and the host-side status check fails the step).
__device__ void raise_abort(const DpArgs& a, int base) {
  __threadfence_system();
  for (int d = 0; d < a.D; ++d) st_volatile(a.flags[d] + kFlagAbort, base + 3);
  __threadfence_system();
}

// Wait until flags[idx(d)] >= epoch for every rank d (in our own page).  Returns false on
// timeout (after raising the abort mark in every page) or when a peer raised it.
__device__ bool wait_all_flags(const DpArgs& a, int epoch, int base) {
  const int* own = a.flags[a.rank];
  const uint64_t t0 = globaltimer_ns();
  for (int d = 0; d < a.D; ++d) {
    while (ld_volatile(own + kFlagEpoch + d) < epoch) {
      if (aborted(own, base)) {
        atomicOr(a.status, kStatusFlagTimeout);
        return false;
      }
      if (globaltimer_ns() - t0 > static_cast<uint64_t>(a.timeout_ns)) {
        atomicOr(a.status, kStatusFlagTimeout);
        raise_abort(a, base);
        return false;
      }
      __nanosleep(256);
    }
  }
  __threadfence_system();
  return true;
}

__global__ void __launch_bounds__(512, 2) dp_reduce_adamw_kernel(DpArgs a) {
  cg::grid_group grid = cg::this_grid();
  __shared__ float red[32];
  __shared__ float s_coef;
  __shared__ int s_ok;
  const long long shard = a.n / a.D;
  const long long lo4 = (a.rank * shard) / 4, hi4 = ((a.rank + 1) * shard) / 4;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long nthreads = static_cast<long long>(gridDim.x) * blockDim.x;
  const int base = 3 * a.epoch;
  // ---- barrier 0: every replica's backward has finished writing its gradients
  if (tid == 0) {
    a.sumsq_scratch[0] = 0.f;
    __threadfence_system();
    for (int d = 0; d < a.D; ++d) st_volatile(a.flags[d] + kFlagEpoch + a.rank, base + 1);
    a.sumsq_scratch[1] = wait_all_flags(a, base + 1, base) ? 1.f : -1.f;
  }
  grid.sync();
  if (reinterpret_cast<volatile float*>(a.sumsq_scratch)[1] < 0.f) return;

  // ---- A: reduce my shard, norm partials.  kU float4 of every replica are in flight per
  // thread before any is used: one remote load per thread at a time left the NVLink reads
  // latency-bound (about 0.4 of the link rate).
  constexpr int kU = 4;
  float acc = 0.f;
  for (long long i0 = lo4 + tid; i0 < hi4; i0 += kU * nthreads) {
    float4 s[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long i = i0 + u * nthreads;
      s[u] = i < hi4 ? reinterpret_cast<const float4*>(a.grad[a.rank])[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int d = 0; d < a.D; ++d) {
      if (d == a.rank) continue;
      float4 g[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const long long i = i0 + u * nthreads;
        g[u] = i < hi4 ? __ldcs(reinterpret_cast<const float4*>(a.grad[d]) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        s[u].x += g[u].x; s[u].y += g[u].y; s[u].z += g[u].z; s[u].w += g[u].w;
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long long i = i0 + u * nthreads;
      if (i >= hi4) break;
      float4 t = s[u];
      t.x *= a.inv_d; t.y *= a.inv_d; t.z *= a.inv_d; t.w *= a.inv_d;
      reinterpret_cast<float4*>(a.grad[a.rank])[i] = t;
      acc += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
    }
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(a.sumsq_scratch, v);
  }
  grid.sync();

  // ---- B: exchange norms, barrier 1
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const float mine = a.sumsq_scratch[0];
    for (int d = 0; d < a.D; ++d) st_volatile(a.flags[d] + kFlagNorm + a.rank, __float_as_int(mine));
    __threadfence_system();
    for (int d = 0; d < a.D; ++d) st_volatile(a.flags[d] + kFlagEpoch + a.rank, base + 2);
    int ok = wait_all_flags(a, base + 2, base) ? 1 : 0;
    // a peer that gave up at barrier 0 or 1 skips its update: then nobody updates
    if (ok && aborted(a.flags[a.rank], base)) {
      atomicOr(a.status, kStatusFlagTimeout);
      ok = 0;
    }
    float total = 0.f;
    for (int d = 0; d < a.D; ++d) total += __int_as_float(ld_volatile(a.flags[a.rank] + kFlagNorm + d));
    float coef = 1.f;
    if (a.max_norm > 0.f) coef = fminf(1.f, a.max_norm / (sqrtf(total) + 1e-6f));
    a.sumsq_scratch[1] = ok ? coef : -1.f;
  }
  grid.sync();
  if (threadIdx.x == 0) {
    const float c = reinterpret_cast<volatile float*>(a.sumsq_scratch)[1];
    s_coef = c;
    s_ok = c >= 0.f;
  }
  __syncthreads();
  if (!s_ok) return;  // a peer never arrived: leave parameters untouched, error is recorded
  const float coef = s_coef;

  // ---- C: AdamW on my shard, broadcast parameters to every replica
  const float decay = 1.f - a.lr * a.wd;
  constexpr int kUC = 2;  // g, p, m, v of kUC float4 in flight (64 registers: two blocks per SM)
  for (long long i0 = lo4 + tid; i0 < hi4; i0 += kUC * nthreads) {
    float4 gg[kUC], p[kUC], m[kUC], v[kUC];
#pragma unroll
    for (int u = 0; u < kUC; ++u) {
      const long long i = i0 + u * nthreads;
      if (i < hi4) {
        gg[u] = reinterpret_cast<const float4*>(a.grad[a.rank])[i];
        p[u] = reinterpret_cast<const float4*>(a.param[a.rank])[i];
        m[u] = reinterpret_cast<const float4*>(a.m)[i];
        v[u] = reinterpret_cast<const float4*>(a.v)[i];
      }
    }
#pragma unroll
    for (int u = 0; u < kUC; ++u) {
      const long long i = i0 + u * nthreads;
      if (i >= hi4) break;
      if (a.zero_grad) reinterpret_cast<float4*>(a.grad[a.rank])[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      const float g4[4] = {gg[u].x * coef, gg[u].y * coef, gg[u].z * coef, gg[u].w * coef};
      float* pp = &p[u].x;
      float* mp = &m[u].x;
      float* vp = &v[u].x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        mp[j] = a.beta1 * mp[j] + (1.f - a.beta1) * g4[j];
        vp[j] = a.beta2 * vp[j] + (1.f - a.beta2) * g4[j] * g4[j];
        pp[j] = pp[j] * decay - a.step_size * mp[j] / (sqrtf(vp[j]) * a.inv_bc2_sqrt + a.eps);
      }
      reinterpret_cast<float4*>(a.m)[i] = m[u];
      reinterpret_cast<float4*>(a.v)[i] = v[u];
      const uint2 sh = make_uint2(pack_bf16x2(p[u].x, p[u].y), pack_bf16x2(p[u].z, p[u].w));
      for (int d = 0; d < a.D; ++d) {
        reinterpret_cast<float4*>(a.param[d])[i] = p[u];
        if (a.shadow[d]) reinterpret_cast<uint2*>(a.shadow[d])[i] = sh;
      }
    }
  }
  if (a.zero_grad) {
    // the rest of this rank's gradient buffer: the peers finished reading it before barrier 1
    const long long n4 = a.n / 4;
    for (long long i = tid; i < n4; i += nthreads) {
      if (i >= lo4 && i < hi4) continue;
      reinterpret_cast<float4*>(a.grad[a.rank])[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  __threadfence_system();
  grid.sync();

  // ---- D: barrier 2 (every replica's parameter stores are visible)
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    __threadfence_system();
    for (int d = 0; d < a.D; ++d) st_volatile(a.flags[d] + kFlagEpoch + a.rank, base + 3);
    wait_all_flags(a, base + 3, base);
  }
}

__global__ void flag_wait_probe_kernel(int* flag, int expect, long long timeout_ns, int* status, int* result) {
  const uint64_t t0 = globaltimer_ns();
  while (ld_volatile(flag) < expect) {
    if (globaltimer_ns() - t0 > static_cast<uint64_t>(timeout_ns)) {
      atomicOr(status, kStatusFlagTimeout);
      *result = -1;
      return;
    }
    __nanosleep(1000);
  }
  *result = 1;
}

// ------------------------------------------------------------------ host side
void dp_reduce_adamw(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& param_ptrs,
                     const std::vector<int64_t>& shadow_ptrs, const std::vector<int64_t>& flag_ptrs, torch::Tensor m,
                     torch::Tensor v, torch::Tensor scratch, int64_t n, int64_t rank, int64_t epoch, double lr,
                     double beta1, double beta2, double eps, double wd, int64_t step, double max_norm,
                     double timeout_s, bool zero_grad) {
  const int D = static_cast<int>(grad_ptrs.size());
  REVPP_CHECK(D >= 1 && D <= kMaxPeers, "1..8 replicas");
  REVPP_CHECK(param_ptrs.size() == static_cast<size_t>(D) && flag_ptrs.size() == static_cast<size_t>(D),
              "one pointer per replica");
  REVPP_CHECK(n % (4 * D) == 0, "flat size must be a multiple of 4 * replicas");
  check_cuda_f32(m, "m");
  check_cuda_f32(v, "v");
  check_cuda_f32(scratch, "scratch");
  c10::cuda::CUDAGuard guard(m.device());
  DpArgs a{};
  for (int d = 0; d < D; ++d) {
    a.grad[d] = reinterpret_cast<float*>(grad_ptrs[d]);
    a.param[d] = reinterpret_cast<float*>(param_ptrs[d]);
    a.shadow[d] = shadow_ptrs.empty() ? nullptr : reinterpret_cast<__nv_bfloat16*>(shadow_ptrs[d]);
    a.flags[d] = reinterpret_cast<int*>(flag_ptrs[d]);
  }
  a.m = m.data_ptr<float>();
  a.v = v.data_ptr<float>();
  a.sumsq_scratch = scratch.data_ptr<float>();
  a.n = n;
  a.D = D;
  a.rank = static_cast<int>(rank);
  a.epoch = static_cast<int>(epoch);
  a.zero_grad = zero_grad ? 1 : 0;
  const double bc1 = 1.0 - std::pow(beta1, static_cast<double>(step));
  const double bc2 = 1.0 - std::pow(beta2, static_cast<double>(step));
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.wd = static_cast<float>(wd);
  a.step_size = static_cast<float>(lr / bc1);
  a.inv_bc2_sqrt = static_cast<float>(1.0 / std::sqrt(bc2));
  a.max_norm = static_cast<float>(max_norm);
  a.inv_d = 1.f / D;
  a.timeout_ns = static_cast<long long>(timeout_s * 1e9);
  a.status = status_device_ptr();
  int per_sm = 0;
  REVPP_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dp_reduce_adamw_kernel, 512, 0));
  REVPP_CHECK(per_sm >= 1, "dp kernel cannot be resident");
  const int grid = std::max(1, std::min(per_sm, 2) * gemm_grid_sms());
  void* params[] = {&a};
  REVPP_CUDA_CHECK(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(dp_reduce_adamw_kernel), dim3(grid), dim3(512),
                                               params, 0, cur_stream()));
  count_launch();
}

// Map a peer's allocation (CUDA IPC handle bytes) into this process *for the current
// device*, with lazy peer access; returns the base address.  The mapping must be made
// with the consuming GPU current: torch's own storage sharing opens handles under the
// producer's device index, which maps the memory for the wrong GPU in a multi-GPU
// process group (a kernel on this GPU then faults on the address).
int64_t ipc_open(const std::string& handle_bytes) {
  REVPP_CHECK(handle_bytes.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size ", handle_bytes.size());
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle_bytes.data(), sizeof(h));
  void* p = nullptr;
  REVPP_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  // the owner GPU must be reachable from the current one: peer access enabled (lazily by
  // the open above, or already) or the same device
  int cur = -1;
  REVPP_CUDA_CHECK(cudaGetDevice(&cur));
  cudaPointerAttributes attr;
  REVPP_CUDA_CHECK(cudaPointerGetAttributes(&attr, p));
  if (attr.device != cur) {
    int can = 0;
    REVPP_CUDA_CHECK(cudaDeviceCanAccessPeer(&can, cur, attr.device));
    if (!can) {
      cudaIpcCloseMemHandle(p);
      REVPP_CHECK(false, "GPU ", cur, " cannot access peer GPU ", attr.device);
    }
    const cudaError_t e = cudaDeviceEnablePeerAccess(attr.device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
      cudaGetLastError();
    } else if (e != cudaSuccess) {
      cudaIpcCloseMemHandle(p);
      REVPP_CHECK(false, "enabling peer access ", cur, " -> ", attr.device, ": ", cudaGetErrorString(e));
    }
  }
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t base) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(base)); }

// Copy a contiguous CUDA tensor to a device address on the current stream.  For an address
// in a peer GPU's IPC-mapped memory this is a copy-engine transfer over NVLink: it uses no
// SMs, so it overlaps the kernels of both GPUs (the pipeline's stage-to-stage messages).
void copy_to_ptr(int64_t dst, const torch::Tensor& src) {
  REVPP_CHECK(src.is_cuda() && src.is_contiguous(), "copy_to_ptr needs a contiguous CUDA tensor");
  REVPP_CHECK(dst != 0 && (dst & 15) == 0, "destination must be a 16-byte aligned device address");
  c10::cuda::CUDAGuard guard(src.device());
  REVPP_CUDA_CHECK(cudaMemcpyAsync(reinterpret_cast<void*>(dst), src.data_ptr(), src.nbytes(),
                                   cudaMemcpyDeviceToDevice, cur_stream()));
}

// IPC handle bytes and byte offset of the allocation containing `t`'s data.
std::vector<std::string> ipc_export(const torch::Tensor& t) {
  REVPP_CHECK(t.is_cuda(), "IPC export needs a CUDA tensor");
  c10::cuda::CUDAGuard guard(t.device());
  void* ptr = t.data_ptr();
  CUdeviceptr base = 0;
  size_t size = 0;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  REVPP_CUDA_CHECK(cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q));
  REVPP_CHECK(q == cudaDriverEntryPointSuccess && fn != nullptr, "cuMemGetAddressRange unavailable");
  using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  const CUresult r = reinterpret_cast<Fn>(fn)(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  REVPP_CHECK(r == CUDA_SUCCESS, "cuMemGetAddressRange failed ", static_cast<int>(r));
  cudaIpcMemHandle_t h;
  REVPP_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  const int64_t off = reinterpret_cast<int64_t>(ptr) - static_cast<int64_t>(base);
  return {std::string(reinterpret_cast<const char*>(&h), sizeof(h)), std::to_string(off)};
}

// (memory type, device ordinal) of a device pointer as the driver sees it: used to check
// peer mappings before any kernel dereferences them.
std::vector<int64_t> pointer_info(int64_t ptr) {
  cudaPointerAttributes attr;
  const cudaError_t e = cudaPointerGetAttributes(&attr, reinterpret_cast<const void*>(ptr));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return {-1, -1};
  }
  return {static_cast<int64_t>(attr.type), static_cast<int64_t>(attr.device)};
}

// Waits (one thread) until *flag >= expect or the time limit passes; result[0] = 1 or -1.
void flag_wait_probe(torch::Tensor flag, int64_t expect, double timeout_s, torch::Tensor result) {
  REVPP_CHECK(flag.is_cuda() && flag.scalar_type() == at::kInt, "flag must be an int32 CUDA tensor");
  REVPP_CHECK(result.is_cuda() && result.scalar_type() == at::kInt, "result must be an int32 CUDA tensor");
  c10::cuda::CUDAGuard guard(flag.device());
  flag_wait_probe_kernel<<<1, 1, 0, cur_stream()>>>(flag.data_ptr<int>(), static_cast<int>(expect),
                                                    static_cast<long long>(timeout_s * 1e9), status_device_ptr(),
                                                    result.data_ptr<int>());
  REVPP_CHECK_LAUNCH();
}

}  // namespace revpp
