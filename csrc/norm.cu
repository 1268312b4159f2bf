// LayerNorm forward / backward and the small reductions that ride along.
//
// Forward : y = (x - mean) * rstd * gamma + beta, x fp32 [M, H], y bf16 or fp32.
//           One warp per row, the row lives in registers (two-pass variance).
// Backward: dx = rstd * (g - mean(g) - xhat * mean(g * xhat)), g = dy * gamma,
//           with dgamma += sum(dy * xhat), dbeta += sum(dy) and, fused:
//             dx_out = dx + resid_grad            (reversible gradient add)
//             dx_bf16 = bf16(dx_out)               (next GEMM operand)
//             colsum += sum_rows(dx_out)          (bias gradient of the producer)
//
// Replaces ATen layer_norm (BERT/models/bert_blocks.py:35-63, autocast runs it in fp32).
#include "common.cuh"
#include "host.h"

namespace revpp {

constexpr int kLnWarps = 8;

template <int VPL>  // float4 per lane, H = VPL * 128
__global__ void __launch_bounds__(kLnWarps * 32)
    ln_fwd_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ gamma,
                  const float* __restrict__ beta, float eps, int M, __nv_bfloat16* __restrict__ y_bf16,
                  float* __restrict__ y_f32, float* __restrict__ y2_f32, long long ldy, float* __restrict__ mean_out,
                  float* __restrict__ rstd_out) {
  constexpr int H = VPL * 128;
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= M) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<long long>(row) * ldx);
  float4 v[VPL];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    v[i] = xr[lane + 32 * i];
    s += v[i].x + v[i].y + v[i].z + v[i].w;
  }
  const float mean = warp_sum(s) * (1.0f / H);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    ss += a * a + b * b + c * c + d * d;
  }
  const float var = warp_sum(ss) * (1.0f / H);
  const float rstd = rsqrtf(var + eps);
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c4 = lane + 32 * i;
    const float4 g = __ldg(g4 + c4), b = __ldg(b4 + c4);
    float4 o;
    o.x = (v[i].x - mean) * rstd * g.x + b.x;
    o.y = (v[i].y - mean) * rstd * g.y + b.y;
    o.z = (v[i].z - mean) * rstd * g.z + b.z;
    o.w = (v[i].w - mean) * rstd * g.w + b.w;
    const long long off = static_cast<long long>(row) * ldy + 4 * c4;
    if (y_bf16) {
      uint2 p = make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
      *reinterpret_cast<uint2*>(y_bf16 + off) = p;
    }
    if (y_f32) *reinterpret_cast<float4*>(y_f32 + off) = o;
    if (y2_f32) *reinterpret_cast<float4*>(y2_f32 + off) = o;
  }
}

// One warp per row.  The per-column sums (dgamma, dbeta, column sum of dx) accumulate in
// a per-warp shared-memory slice (each lane owns its columns, so no atomics) instead of
// 3 x 4 x VPL registers per lane: that keeps the kernel at about 128 registers, two
// blocks (16 warps) per SM, and lets every lane issue its row's dy / x / residual loads
// together.  The slices are summed per block at the end, one global atomic per column.
template <int VPL, bool DY_BF16>
__global__ void __launch_bounds__(kLnWarps * 32, VPL <= 8 ? 2 : 1)
    ln_bwd_kernel(const void* __restrict__ dy_, long long lddy, const float* __restrict__ x, long long ldx,
                  const float* __restrict__ gamma, const float* __restrict__ mean_in,
                  const float* __restrict__ rstd_in, int M, float* __restrict__ dgamma, float* __restrict__ dbeta,
                  const float* __restrict__ resid, long long ldr, float* __restrict__ dx_f32,
                  __nv_bfloat16* __restrict__ dx_bf16, long long lddx, float* __restrict__ colsum) {
  constexpr int H = VPL * 128;
  extern __shared__ float4 s_acc4[];  // [kLnWarps][3][H / 4]
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const bool want_gb = dgamma != nullptr || dbeta != nullptr;
  const bool want_cs = colsum != nullptr;
  float4* acc_g = s_acc4 + (warp * 3 + 0) * (H / 4);
  float4* acc_b = s_acc4 + (warp * 3 + 1) * (H / 4);
  float4* acc_c = s_acc4 + (warp * 3 + 2) * (H / 4);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    acc_g[lane + 32 * i] = z;
    acc_b[lane + 32 * i] = z;
    acc_c[lane + 32 * i] = z;
  }
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  for (int row = blockIdx.x * kLnWarps + warp; row < M; row += gridDim.x * kLnWarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<long long>(row) * ldx);
    const float4* rr = resid ? reinterpret_cast<const float4*>(resid + static_cast<long long>(row) * ldr) : nullptr;
    const float mean = mean_in[row], rstd = rstd_in[row];
    float4 dy[VPL], xh[VPL], rv[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c4 = lane + 32 * i;
      if constexpr (DY_BF16) {
        const uint2 p = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(dy_) +
                                                        static_cast<long long>(row) * lddy + 4 * c4);
        const float2 a = unpack_bf16x2(p.x), b = unpack_bf16x2(p.y);
        dy[i] = make_float4(a.x, a.y, b.x, b.y);
      } else {
        dy[i] = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(dy_) + static_cast<long long>(row) * lddy +
                                                 4 * c4);
      }
      xh[i] = xr[c4];
      rv[i] = rr ? rr[c4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const float4 g = __ldg(g4 + lane + 32 * i);
      xh[i] = make_float4((xh[i].x - mean) * rstd, (xh[i].y - mean) * rstd, (xh[i].z - mean) * rstd,
                          (xh[i].w - mean) * rstd);
      const float gx = dy[i].x * g.x, gy = dy[i].y * g.y, gz = dy[i].z * g.z, gw = dy[i].w * g.w;
      s1 += gx + gy + gz + gw;
      s2 += gx * xh[i].x + gy * xh[i].y + gz * xh[i].z + gw * xh[i].w;
    }
    const float m1 = warp_sum(s1) * (1.0f / H);
    const float m2 = warp_sum(s2) * (1.0f / H);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c4 = lane + 32 * i;
      const float4 g = __ldg(g4 + c4);
      float4 d;
      d.x = rstd * (dy[i].x * g.x - m1 - xh[i].x * m2) + rv[i].x;
      d.y = rstd * (dy[i].y * g.y - m1 - xh[i].y * m2) + rv[i].y;
      d.z = rstd * (dy[i].z * g.z - m1 - xh[i].z * m2) + rv[i].z;
      d.w = rstd * (dy[i].w * g.w - m1 - xh[i].w * m2) + rv[i].w;
      const long long off = static_cast<long long>(row) * lddx + 4 * c4;
      if (dx_f32) *reinterpret_cast<float4*>(dx_f32 + off) = d;
      if (dx_bf16) *reinterpret_cast<uint2*>(dx_bf16 + off) = make_uint2(pack_bf16x2(d.x, d.y), pack_bf16x2(d.z, d.w));
      if (want_gb) {
        float4 ag = acc_g[c4], ab = acc_b[c4];
        ag.x += dy[i].x * xh[i].x; ag.y += dy[i].y * xh[i].y; ag.z += dy[i].z * xh[i].z; ag.w += dy[i].w * xh[i].w;
        ab.x += dy[i].x; ab.y += dy[i].y; ab.z += dy[i].z; ab.w += dy[i].w;
        acc_g[c4] = ag;
        acc_b[c4] = ab;
      }
      if (want_cs) {
        float4 ac = acc_c[c4];
        ac.x += d.x; ac.y += d.y; ac.z += d.z; ac.w += d.w;
        acc_c[c4] = ac;
      }
    }
  }
  __syncthreads();
  // one 16-byte vector atomic per 4 columns and block (a scalar atomic per column put
  // four times as many same-line operations in L2's queue)
  for (int c4 = threadIdx.x; c4 < H / 4; c4 += blockDim.x) {
    float4 tg = make_float4(0.f, 0.f, 0.f, 0.f), tb = tg, tc = tg;
#pragma unroll
    for (int w = 0; w < kLnWarps; ++w) {
      const float4 g = s_acc4[(w * 3 + 0) * (H / 4) + c4];
      const float4 b = s_acc4[(w * 3 + 1) * (H / 4) + c4];
      const float4 c = s_acc4[(w * 3 + 2) * (H / 4) + c4];
      tg.x += g.x; tg.y += g.y; tg.z += g.z; tg.w += g.w;
      tb.x += b.x; tb.y += b.y; tb.z += b.z; tb.w += b.w;
      tc.x += c.x; tc.y += c.y; tc.z += c.z; tc.w += c.w;
    }
    if (dgamma) atomicAdd(reinterpret_cast<float4*>(dgamma) + c4, tg);
    if (dbeta) atomicAdd(reinterpret_cast<float4*>(dbeta) + c4, tb);
    if (colsum) atomicAdd(reinterpret_cast<float4*>(colsum) + c4, tc);
  }
}

// out_bf16 = bf16(in_f32) and colsum += sum_rows(in), in fp32 [M, N].
// Or, with a bf16 input, only the column sum.
// Tile = 128 rows x 256 columns per CTA: 64 threads x 4 columns across, 4 row groups
// down; the row groups are reduced in shared memory, so each column sees one atomic per
// 128 rows.
constexpr int kColTileRows = 128;
template <bool IN_BF16>
__global__ void __launch_bounds__(256)
    cast_colsum_kernel(const void* __restrict__ in_, long long ldi, int M, int N, __nv_bfloat16* __restrict__ out,
                       long long ldo, float* __restrict__ colsum) {
  __shared__ float4 red[3][64];
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
  const int c4 = blockIdx.y * 64 + tx;
  const bool col_ok = 4 * c4 < N;
  const int r0 = blockIdx.x * kColTileRows;
  const int r1 = min(M, r0 + kColTileRows);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col_ok) {
    for (int r = r0 + ty; r < r1; r += 4) {
      float4 v;
      if constexpr (IN_BF16) {
        const uint2 p = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(in_) +
                                                        static_cast<long long>(r) * ldi + 4 * c4);
        const float2 a = unpack_bf16x2(p.x), b = unpack_bf16x2(p.y);
        v = make_float4(a.x, a.y, b.x, b.y);
      } else {
        v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(in_) + static_cast<long long>(r) * ldi +
                                             4 * c4);
        if (out) {
          *reinterpret_cast<uint2*>(out + static_cast<long long>(r) * ldo + 4 * c4) =
              make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
        }
      }
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  if (ty > 0) red[ty - 1][tx] = acc;
  __syncthreads();
  if (ty == 0 && col_ok && colsum) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      acc.x += red[k][tx].x; acc.y += red[k][tx].y; acc.z += red[k][tx].z; acc.w += red[k][tx].w;
    }
    atomicAdd(reinterpret_cast<float4*>(colsum) + c4, acc);
  }
}

// ------------------------------------------------------------------ host side
namespace {
template <typename F>
void dispatch_vpl(int H, F&& f) {
  REVPP_CHECK(H % 128 == 0 && H >= 128 && H <= 2048, "LayerNorm width must be a multiple of 128 in [128, 2048], got ",
              H);
  switch (H / 128) {
    case 1: f(std::integral_constant<int, 1>{}); break;
    case 2: f(std::integral_constant<int, 2>{}); break;
    case 3: f(std::integral_constant<int, 3>{}); break;
    case 4: f(std::integral_constant<int, 4>{}); break;
    case 5: f(std::integral_constant<int, 5>{}); break;
    case 6: f(std::integral_constant<int, 6>{}); break;
    case 7: f(std::integral_constant<int, 7>{}); break;
    case 8: f(std::integral_constant<int, 8>{}); break;
    case 12: f(std::integral_constant<int, 12>{}); break;
    case 16: f(std::integral_constant<int, 16>{}); break;
    default: REVPP_CHECK(false, "unsupported LayerNorm width ", H);
  }
}
float* opt_f32(const c10::optional<torch::Tensor>& t) {
  if (!t.has_value() || !t->defined()) return nullptr;
  check_cuda_f32(*t, "tensor");
  return t->data_ptr<float>();
}
}  // namespace

// x fp32 [M, H] (row stride), gamma/beta fp32 [H].  Writes any of y_bf16, y_f32, y2_f32 (same row stride).
void layernorm_fwd(const torch::Tensor& x, const torch::Tensor& gamma, const torch::Tensor& beta, double eps,
                   const c10::optional<torch::Tensor>& y_bf16, const c10::optional<torch::Tensor>& y_f32,
                   const c10::optional<torch::Tensor>& y2_f32, const c10::optional<torch::Tensor>& mean,
                   const c10::optional<torch::Tensor>& rstd) {
  check_cuda_f32(x, "x");
  REVPP_CHECK(x.dim() == 2 && x.stride(1) == 1);
  const int M = static_cast<int>(x.size(0)), H = static_cast<int>(x.size(1));
  c10::cuda::CUDAGuard guard(x.device());
  long long ldy = H;
  __nv_bfloat16* yb = nullptr;
  if (y_bf16.has_value() && y_bf16->defined()) {
    check_cuda_bf16(*y_bf16, "y_bf16");
    yb = reinterpret_cast<__nv_bfloat16*>(y_bf16->data_ptr());
    ldy = y_bf16->stride(0);
  }
  float* yf = opt_f32(y_f32);
  float* yf2 = opt_f32(y2_f32);
  if (yf) ldy = y_f32->stride(0);
  if (yb && yf) REVPP_CHECK(y_f32->stride(0) == ldy, "outputs must share the row stride");
  if (yf2) REVPP_CHECK(y2_f32->stride(0) == ldy, "outputs must share the row stride");
  const int grid = (M + kLnWarps - 1) / kLnWarps;
  if (M == 0) return;
  dispatch_vpl(H, [&](auto vpl) {
    launch_pdl(ln_fwd_kernel<decltype(vpl)::value>, dim3(grid), dim3(kLnWarps * 32), 0, cur_stream(),
        x.data_ptr<float>(), x.stride(0), gamma.data_ptr<float>(), beta.data_ptr<float>(), static_cast<float>(eps), M,
        yb, yf, yf2, ldy, opt_f32(mean), opt_f32(rstd));
  });
  REVPP_CHECK_LAUNCH();
}

// dy (bf16 or fp32) [M, H]; returns through dx_f32 / dx_bf16 (shared row stride).
void layernorm_bwd(const torch::Tensor& dy, const torch::Tensor& x, const torch::Tensor& gamma,
                   const torch::Tensor& mean, const torch::Tensor& rstd, const c10::optional<torch::Tensor>& dgamma,
                   const c10::optional<torch::Tensor>& dbeta, const c10::optional<torch::Tensor>& resid,
                   const c10::optional<torch::Tensor>& dx_f32, const c10::optional<torch::Tensor>& dx_bf16,
                   const c10::optional<torch::Tensor>& colsum) {
  check_cuda_f32(x, "x");
  REVPP_CHECK(dy.dim() == 2 && dy.stride(1) == 1 && x.stride(1) == 1);
  const int M = static_cast<int>(x.size(0)), H = static_cast<int>(x.size(1));
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  const bool dy_bf16 = dy.scalar_type() == at::kBFloat16;
  for (const auto* t : {&dgamma, &dbeta, &colsum}) {  // the column sums use 16-byte vector atomics
    if (t->has_value() && (*t)->defined()) {
      REVPP_CHECK((*t)->numel() >= H && (reinterpret_cast<uintptr_t>((*t)->data_ptr()) & 15) == 0,
                  "LayerNorm backward gradient sums need 16-byte aligned fp32 buffers of H elements");
    }
  }
  float* dxf = opt_f32(dx_f32);
  __nv_bfloat16* dxb = nullptr;
  long long lddx = H;
  if (dxf) lddx = dx_f32->stride(0);
  if (dx_bf16.has_value() && dx_bf16->defined()) {
    check_cuda_bf16(*dx_bf16, "dx_bf16");
    dxb = reinterpret_cast<__nv_bfloat16*>(dx_bf16->data_ptr());
    if (dxf) REVPP_CHECK(dx_bf16->stride(0) == lddx, "dx outputs must share the row stride");
    lddx = dx_bf16->stride(0);
  }
  const float* rp = opt_f32(resid);
  const long long ldr = rp ? resid->stride(0) : 0;
  const int grid = std::min((M + kLnWarps - 1) / kLnWarps, 2 * num_sms());
  dispatch_vpl(H, [&](auto vpl) {
    constexpr int V = decltype(vpl)::value;
    const int smem = kLnWarps * 3 * V * 128 * static_cast<int>(sizeof(float));
    static int configured_for[2] = {-1, -1};
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_for[dy_bf16] != dev) {
      if (dy_bf16) {
        REVPP_CUDA_CHECK(cudaFuncSetAttribute(ln_bwd_kernel<V, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      } else {
        REVPP_CUDA_CHECK(cudaFuncSetAttribute(ln_bwd_kernel<V, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      }
      configured_for[dy_bf16] = dev;
    }
    if (dy_bf16) {
      launch_pdl(ln_bwd_kernel<V, true>, dim3(grid), dim3(kLnWarps * 32), smem, cur_stream(),
          dy.data_ptr(), dy.stride(0), x.data_ptr<float>(), x.stride(0), gamma.data_ptr<float>(), mean.data_ptr<float>(),
          rstd.data_ptr<float>(), M, opt_f32(dgamma), opt_f32(dbeta), rp, ldr, dxf, dxb, lddx, opt_f32(colsum));
    } else {
      launch_pdl(ln_bwd_kernel<V, false>, dim3(grid), dim3(kLnWarps * 32), smem, cur_stream(),
          dy.data_ptr(), dy.stride(0), x.data_ptr<float>(), x.stride(0), gamma.data_ptr<float>(), mean.data_ptr<float>(),
          rstd.data_ptr<float>(), M, opt_f32(dgamma), opt_f32(dbeta), rp, ldr, dxf, dxb, lddx, opt_f32(colsum));
    }
  });
  REVPP_CHECK_LAUNCH();
}

// fp32 in: out = bf16(in) (optional) and colsum += column sums (optional).  bf16 in: colsum only.
void cast_colsum(const torch::Tensor& in, const c10::optional<torch::Tensor>& out,
                 const c10::optional<torch::Tensor>& colsum) {
  REVPP_CHECK(in.is_cuda() && in.dim() == 2 && in.stride(1) == 1, "input must be a 2-D CUDA tensor, unit inner stride");
  const int M = static_cast<int>(in.size(0)), N = static_cast<int>(in.size(1));
  REVPP_CHECK(N % 4 == 0, "cast_colsum needs N % 4 == 0");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(in.device());
  __nv_bfloat16* op = nullptr;
  long long ldo = N;
  if (out.has_value() && out->defined()) {
    check_cuda_bf16(*out, "out");
    op = reinterpret_cast<__nv_bfloat16*>(out->data_ptr());
    ldo = out->stride(0);
  }
  float* cs = opt_f32(colsum);
  REVPP_CHECK(cs == nullptr || (reinterpret_cast<uintptr_t>(cs) & 15) == 0,
              "cast_colsum: colsum must be 16-byte aligned (vector atomics)");
  dim3 grid((M + kColTileRows - 1) / kColTileRows, (N / 4 + 63) / 64);
  if (in.scalar_type() == at::kBFloat16) {
    cast_colsum_kernel<true><<<grid, 256, 0, cur_stream()>>>(in.data_ptr(), in.stride(0), M, N, nullptr, 0, cs);
  } else {
    check_cuda_f32(in, "in");
    cast_colsum_kernel<false><<<grid, 256, 0, cur_stream()>>>(in.data_ptr(), in.stride(0), M, N, op, ldo, cs);
  }
  REVPP_CHECK_LAUNCH();
}

}  // namespace revpp
