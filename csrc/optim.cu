// Gradient norm and fused AdamW over a stage's flat parameter buffers.
//
//   sumsq_accumulate : out[0] += sum(g^2)                       (grad-norm pass)
//   adamw_fused      : coef = min(1, max_norm / (sqrt(sumsq) + 1e-6))   (clip_grad_norm_)
//                      g' = g * coef
//                      p  = p * (1 - lr * wd)
//                      m  = b1 m + (1 - b1) g'
//                      v  = b2 v + (1 - b2) g'^2
//                      p -= (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps)
//                      shadow = bf16(p), g = 0
// One read and one write of every buffer per step; the clip coefficient is read on the
// device, so there is no host synchronisation between the norm and the update.
//
// Replaces torch.nn.utils.clip_grad_norm_ + torch.optim.AdamW (BERT/src/engine.py:56-67,
// BERT/experiment/base.py:303).
#include "common.cuh"
#include "host.h"

namespace revpp {

__global__ void sumsq_kernel(const float4* __restrict__ g, long long n4, float* __restrict__ out) {
  float acc = 0.f;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 v = g[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  acc = warp_sum(acc);
  __shared__ float s[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) s[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    acc = lane < (blockDim.x >> 5) ? s[lane] : 0.f;
    acc = warp_sum(acc);
    if (lane == 0) atomicAdd(out, acc);
  }
}

__global__ void adamw_kernel(float4* __restrict__ p, float4* __restrict__ g, float4* __restrict__ m,
                             float4* __restrict__ v, uint2* __restrict__ shadow, long long n4, float lr, float beta1,
                             float beta2, float eps, float wd, float step_size, float inv_bc2_sqrt, float max_norm,
                             const float* __restrict__ sumsq, int zero_grad) {
  float coef = 1.f;
  if (sumsq != nullptr && max_norm > 0.f) {
    const float norm = sqrtf(*sumsq);
    coef = fminf(1.f, max_norm / (norm + 1e-6f));
  }
  const float decay = 1.f - lr * wd;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 gg = g[i], pp = p[i], mm = m[i], vv = v[i];
    float* gp = &gg.x;
    float* ppp = &pp.x;
    float* mp = &mm.x;
    float* vp = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gj = gp[j] * coef;
      mp[j] = beta1 * mp[j] + (1.f - beta1) * gj;
      vp[j] = beta2 * vp[j] + (1.f - beta2) * gj * gj;
      const float denom = sqrtf(vp[j]) * inv_bc2_sqrt + eps;
      ppp[j] = ppp[j] * decay - step_size * mp[j] / denom;
    }
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    if (shadow) shadow[i] = make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w));
    if (zero_grad) g[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

__global__ void scale_kernel(float4* __restrict__ x, long long n4, float s) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 v = x[i];
    v.x *= s; v.y *= s; v.z *= s; v.w *= s;
    x[i] = v;
  }
}

static int grid_for(long long n4, int threads) {
  const long long want = (n4 + threads - 1) / threads;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(want, 8LL * num_sms())));
}

void grad_sumsq(const torch::Tensor& g, torch::Tensor out) {
  check_cuda_f32(g, "g");
  check_cuda_f32(out, "out");
  REVPP_CHECK(g.is_contiguous() && g.numel() % 4 == 0, "flat grad must be contiguous, numel % 4 == 0");
  c10::cuda::CUDAGuard guard(g.device());
  const long long n4 = g.numel() / 4;
  sumsq_kernel<<<grid_for(n4, 256), 256, 0, cur_stream()>>>(reinterpret_cast<const float4*>(g.data_ptr<float>()), n4,
                                                             out.data_ptr<float>());
  REVPP_CHECK_LAUNCH();
}

void adamw_step(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v,
                const c10::optional<torch::Tensor>& shadow, double lr, double beta1, double beta2, double eps,
                double wd, int64_t step, double max_norm, const c10::optional<torch::Tensor>& sumsq,
                bool zero_grad) {
  for (auto* t : {&p, &g, &m, &v}) {
    check_cuda_f32(*t, "adam buffer");
    REVPP_CHECK(t->is_contiguous() && t->numel() == p.numel(), "adam buffers must be contiguous and equal size");
  }
  REVPP_CHECK(p.numel() % 4 == 0, "numel % 4 == 0");
  REVPP_CHECK(step >= 1, "step counts from 1");
  uint2* sh = nullptr;
  if (shadow.has_value() && shadow->defined()) {
    check_cuda_bf16(*shadow, "shadow");
    REVPP_CHECK(shadow->numel() == p.numel(), "shadow size");
    sh = reinterpret_cast<uint2*>(shadow->data_ptr());
  }
  const float* ss = nullptr;
  if (sumsq.has_value() && sumsq->defined()) {
    check_cuda_f32(*sumsq, "sumsq");
    ss = sumsq->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(p.device());
  const double bc1 = 1.0 - std::pow(beta1, static_cast<double>(step));
  const double bc2 = 1.0 - std::pow(beta2, static_cast<double>(step));
  const float step_size = static_cast<float>(lr / bc1);
  const float inv_bc2_sqrt = static_cast<float>(1.0 / std::sqrt(bc2));
  const long long n4 = p.numel() / 4;
  adamw_kernel<<<grid_for(n4, 256), 256, 0, cur_stream()>>>(
      reinterpret_cast<float4*>(p.data_ptr<float>()), reinterpret_cast<float4*>(g.data_ptr<float>()),
      reinterpret_cast<float4*>(m.data_ptr<float>()), reinterpret_cast<float4*>(v.data_ptr<float>()), sh, n4,
      static_cast<float>(lr), static_cast<float>(beta1), static_cast<float>(beta2), static_cast<float>(eps),
      static_cast<float>(wd), step_size, inv_bc2_sqrt, static_cast<float>(max_norm), ss, zero_grad ? 1 : 0);
  REVPP_CHECK_LAUNCH();
}

void scale_(torch::Tensor x, double s) {
  check_cuda_f32(x, "x");
  REVPP_CHECK(x.is_contiguous() && x.numel() % 4 == 0, "contiguous, numel % 4 == 0");
  c10::cuda::CUDAGuard guard(x.device());
  const long long n4 = x.numel() / 4;
  scale_kernel<<<grid_for(n4, 256), 256, 0, cur_stream()>>>(reinterpret_cast<float4*>(x.data_ptr<float>()), n4,
                                                             static_cast<float>(s));
  REVPP_CHECK_LAUNCH();
}

}  // namespace revpp
