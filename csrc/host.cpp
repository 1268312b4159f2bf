// Host helpers: status word, device properties, TMA descriptor encoding.
#include "host.h"

#include <cstdlib>

#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

namespace revpp {

namespace {
constexpr int kMaxDevices = 64;
int* g_status_host[kMaxDevices] = {nullptr};
int* g_status_dev[kMaxDevices] = {nullptr};
std::mutex g_status_mu;

int current_device() {
  int d = 0;
  REVPP_CUDA_CHECK(cudaGetDevice(&d));
  return d;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    REVPP_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    REVPP_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}
}  // namespace

int* status_device_ptr() {
  const int d = current_device();
  REVPP_CHECK(d < kMaxDevices, "device index too large");
  if (g_status_dev[d]) return g_status_dev[d];
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!g_status_dev[d]) {
    int* h = nullptr;
    REVPP_CUDA_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&h), 64 * sizeof(int),
                                   cudaHostAllocMapped | cudaHostAllocPortable));
    for (int i = 0; i < 64; ++i) h[i] = 0;
    int* dp = nullptr;
    REVPP_CUDA_CHECK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&dp), h, 0));
    g_status_host[d] = h;
    g_status_dev[d] = dp;
  }
  return g_status_dev[d];
}

int status_peek() {
  status_device_ptr();
  return *reinterpret_cast<volatile int*>(g_status_host[current_device()]);
}

int status_read_and_clear() {
  status_device_ptr();
  volatile int* h = g_status_host[current_device()];
  const int v = *h;
  *h = 0;
  return v;
}

namespace {
int g_sm_reserve = 0;
std::atomic<int64_t> g_launches{0};
}
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
int64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }
void set_sm_reserve(int n) { g_sm_reserve = n < 0 ? 0 : n; }
int sm_reserve() { return g_sm_reserve; }

int gemm_grid_sms() {
  const int n = num_sms() - g_sm_reserve;
  return n < 1 ? 1 : n;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("REVPP_PDL");
    return e == nullptr || std::atoi(e) != 0;
  }();
  return on;
}

int num_sms() {
  static int cached[kMaxDevices] = {0};
  const int d = current_device();
  if (!cached[d]) REVPP_CUDA_CHECK(cudaDeviceGetAttribute(&cached[d], cudaDevAttrMultiProcessorCount, d));
  return cached[d];
}

int max_smem_optin() {
  static int cached[kMaxDevices] = {0};
  const int d = current_device();
  if (!cached[d]) REVPP_CUDA_CHECK(cudaDeviceGetAttribute(&cached[d], cudaDevAttrMaxSharedMemoryPerBlockOptin, d));
  return cached[d];
}

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                         uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle) {
  REVPP_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  REVPP_CHECK(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes, got ",
              row_stride_bytes);
  REVPP_CHECK((box_inner * elem_bytes) % 16 == 0, "TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  REVPP_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r), " (inner=", inner,
              " outer=", outer, " stride=", row_stride_bytes, " box=", box_inner, "x", box_outer, ")");
  return m;
}

}  // namespace revpp
