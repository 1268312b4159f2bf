// Embedding, patch-embedding and classifier-head kernels.
//
// BERT embedding (BERT/models/bert_blocks.py:9-31):
//   fwd: x[t] = LN_1e-5(word[id[t]] + pos[t % S] + type[tt[t]])                 fp32 out
//   bwd: recompute the pre-LN sum, LN backward of dx = dX2 + dX1 (the coupling
//        duplicates x), scatter into the word table (padding row 0 skipped), and per
//        position / per type / gamma / beta sums.  One CTA per position owns dpos[s].
// ViT patch embedding (Vit/models/vit_blocks.py:42-62), conv k = s = p as a GEMM:
//   im2col : images fp32 NCHW -> patches bf16 [B*np, C*p*p] (c, kh, kw order = conv weight)
//   GEMM   : conv = patches @ W^T + b  (tcgen05 GEMM, bf16 out as under autocast)
//   assemble fwd: x[b,0] = LN(cls + pos[0]), x[b,1+i] = LN(conv[b,i] + pos[1+i])
//   assemble bwd: LN backward; dcls, dpos sums; dconv (bf16) for the weight-gradient GEMM
// Classifier head (BERT/models/bert_stages.py:436-444, Vit/models/vit_stages.py:410-419):
//   pool   : z = decouple(Y2, Y1) (sum, or concat [Y1, Y2] for the inverse variant),
//            mean over the sequence or the CLS row
//   head   : h = LN(pooled); logits = bf16(bf16(h) W^T + b); CE in fp32; dlogits scaled
//            by grad_scale / batch; dh = dlogits W; LN backward -> dpooled
//   wgrad  : dW += dlogits^T bf16(h), db += sum(dlogits)
//   spread : dY = dpooled / S on every row (mean) or on row 0 (CLS)
#include "common.cuh"
#include "host.h"

namespace revpp {

namespace {
constexpr int kWarps = 8;

template <int VPL>
__device__ __forceinline__ void row_stats(const float4 (&v)[VPL], float& mean, float& rstd, float eps) {
  constexpr int H = VPL * 128;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) s += v[i].x + v[i].y + v[i].z + v[i].w;
  mean = warp_sum(s) * (1.0f / H);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    ss += a * a + b * b + c * c + d * d;
  }
  rstd = rsqrtf(warp_sum(ss) * (1.0f / H) + eps);
}

__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
}  // namespace

// ------------------------------------------------------------------ BERT embedding
template <int VPL>
__global__ void __launch_bounds__(kWarps * 32)
    bert_embed_fwd_kernel(const int64_t* __restrict__ ids, const int64_t* __restrict__ tt,
                          const float* __restrict__ word, const float* __restrict__ pos,
                          const float* __restrict__ type, const float* __restrict__ gamma,
                          const float* __restrict__ beta, float eps, int M, int S, int V, int T,
                          float* __restrict__ out, int* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= M) return;
  constexpr int H = VPL * 128;
  long long id = ids[row];
  long long ty = tt[row];
  if (id < 0 || id >= V || ty < 0 || ty >= T) {  // out-of-range token: record and embed zero
    if (lane == 0) atomicOr(status, kStatusBadShape);
    id = id < 0 || id >= V ? 0 : id;
    ty = ty < 0 || ty >= T ? 0 : ty;
  }
  const int s = row % S;
  const float4* w4 = reinterpret_cast<const float4*>(word + id * H);
  const float4* p4 = reinterpret_cast<const float4*>(pos + static_cast<long long>(s) * H);
  const float4* t4 = reinterpret_cast<const float4*>(type + ty * H);
  float4 v[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) v[i] = f4add(f4add(__ldg(w4 + lane + 32 * i), __ldg(p4 + lane + 32 * i)), __ldg(t4 + lane + 32 * i));
  float mean, rstd;
  row_stats<VPL>(v, mean, rstd, eps);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  float4* o4 = reinterpret_cast<float4*>(out + static_cast<long long>(row) * H);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    const float4 g = __ldg(g4 + c), b = __ldg(b4 + c);
    o4[c] = make_float4((v[i].x - mean) * rstd * g.x + b.x, (v[i].y - mean) * rstd * g.y + b.y,
                        (v[i].z - mean) * rstd * g.z + b.z, (v[i].w - mean) * rstd * g.w + b.w);
  }
}

// grid = S (one CTA per position), 8 warps.  The batch rows of the position are taken 8 at a
// time, one per warp: the warp computes its row's LayerNorm input gradient dv (the gradient
// of the word, position and type rows), dy * x-hat and dy, adds dv to the token's word row
// (float4 atomics in global memory: rows of different tokens), and stores the three rows in
// shared memory; then every thread sums its columns over the 8 rows into registers (dpos,
// dgamma, dbeta, and dtype of each row's type).  No shared-memory atomics: with every warp
// adding into the same columns they serialised (101 us for 16 x 512 rows, 0.21 of HBM).
// type_vocab_size <= kEmbedMaxTypes.
constexpr int kEmbedMaxTypes = 4;
template <int VPL>
__global__ void __launch_bounds__(kWarps * 32)
    bert_embed_bwd_kernel(const int64_t* __restrict__ ids, const int64_t* __restrict__ tt,
                          const float* __restrict__ word, const float* __restrict__ pos,
                          const float* __restrict__ type, const float* __restrict__ gamma, float eps, int B, int S,
                          int V, int T, const float* __restrict__ dx2, const float* __restrict__ dx1,
                          float* __restrict__ dword, float* __restrict__ dpos, float* __restrict__ dtype,
                          float* __restrict__ dgamma, float* __restrict__ dbeta) {
  constexpr int H = VPL * 128;
  constexpr int NT = kWarps * 32;
  constexpr int J = (H + NT - 1) / NT;  // columns per thread
  extern __shared__ float4 sbuf4[];     // [3][kWarps][H / 4]: dv, dy * x-hat, dy of the chunk's rows
  __shared__ int sty[kWarps];
  float* sbuf = reinterpret_cast<float*>(sbuf4);
  const int s = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  float apos[J], ag[J], ab[J], at[kEmbedMaxTypes][J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    apos[j] = ag[j] = ab[j] = 0.f;
#pragma unroll
    for (int t = 0; t < kEmbedMaxTypes; ++t) at[t][j] = 0.f;
  }
  for (int b0 = 0; b0 < B; b0 += kWarps) {
    const int b = b0 + warp;
    if (b < B) {
      const long long row = static_cast<long long>(b) * S + s;
      long long id = ids[row], ty = tt[row];
      id = id < 0 || id >= V ? 0 : id;
      ty = ty < 0 || ty >= T ? 0 : ty;
      const float4* w4 = reinterpret_cast<const float4*>(word + id * H);
      const float4* p4 = reinterpret_cast<const float4*>(pos + static_cast<long long>(s) * H);
      const float4* t4 = reinterpret_cast<const float4*>(type + ty * H);
      float4 v[VPL], dy[VPL];
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int c = lane + 32 * i;
        v[i] = f4add(f4add(__ldg(w4 + c), __ldg(p4 + c)), __ldg(t4 + c));
        dy[i] = reinterpret_cast<const float4*>(dx2 + row * H)[c];
        if (dx1) dy[i] = f4add(dy[i], reinterpret_cast<const float4*>(dx1 + row * H)[c]);
      }
      float mean, rstd;
      row_stats<VPL>(v, mean, rstd, eps);
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const float4 g = __ldg(g4 + lane + 32 * i);
        v[i] = make_float4((v[i].x - mean) * rstd, (v[i].y - mean) * rstd, (v[i].z - mean) * rstd,
                           (v[i].w - mean) * rstd);
        s1 += dy[i].x * g.x + dy[i].y * g.y + dy[i].z * g.z + dy[i].w * g.w;
        s2 += dy[i].x * g.x * v[i].x + dy[i].y * g.y * v[i].y + dy[i].z * g.z * v[i].z + dy[i].w * g.w * v[i].w;
      }
      const float m1 = warp_sum(s1) * (1.0f / H), m2 = warp_sum(s2) * (1.0f / H);
      float4* wrow = reinterpret_cast<float4*>(dword + id * H);
      float4* r_dv = sbuf4 + (0 * kWarps + warp) * (H / 4);
      float4* r_dx = sbuf4 + (1 * kWarps + warp) * (H / 4);
      float4* r_dy = sbuf4 + (2 * kWarps + warp) * (H / 4);
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int c4 = lane + 32 * i;
        const float4 g = __ldg(g4 + c4);
        const float4 dv = make_float4(rstd * (dy[i].x * g.x - m1 - v[i].x * m2), rstd * (dy[i].y * g.y - m1 - v[i].y * m2),
                                      rstd * (dy[i].z * g.z - m1 - v[i].z * m2), rstd * (dy[i].w * g.w - m1 - v[i].w * m2));
        if (id != 0) atomicAdd(wrow + c4, dv);
        r_dv[c4] = dv;
        r_dx[c4] = make_float4(dy[i].x * v[i].x, dy[i].y * v[i].y, dy[i].z * v[i].z, dy[i].w * v[i].w);
        r_dy[c4] = dy[i];
      }
      if (lane == 0) sty[warp] = static_cast<int>(ty);
    }
    __syncthreads();
    const int nr = min(kWarps, B - b0);
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = threadIdx.x + NT * j;
      if (c < H) {
        for (int r = 0; r < nr; ++r) {
          const float d = sbuf[(0 * kWarps + r) * H + c];
          apos[j] += d;
          ag[j] += sbuf[(1 * kWarps + r) * H + c];
          ab[j] += sbuf[(2 * kWarps + r) * H + c];
          const int ty = sty[r];
#pragma unroll
          for (int t = 0; t < kEmbedMaxTypes; ++t)
            if (ty == t) at[t][j] += d;
        }
      }
    }
    __syncthreads();  // the buffers are rewritten by the next chunk
  }
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = threadIdx.x + NT * j;
    if (c >= H) continue;
    dpos[static_cast<long long>(s) * H + c] += apos[j];  // this CTA owns row s
    atomicAdd(dgamma + c, ag[j]);
    atomicAdd(dbeta + c, ab[j]);
#pragma unroll
    for (int t = 0; t < kEmbedMaxTypes; ++t)
      if (t < T && at[t][j] != 0.f) atomicAdd(dtype + static_cast<long long>(t) * H + c, at[t][j]);
  }
}

// ------------------------------------------------------------------ ViT patch embedding
// patches[b*np + py*g + px, c*p*p + kh*p + kw] = bf16(img[b, c, py*p + kh, px*p + kw])
__global__ void im2col_patches_kernel(const float* __restrict__ img, __nv_bfloat16* __restrict__ out, int B, int C,
                                      int I, int p) {
  const int g = I / p, np = g * g, K = C * p * p;
  const long long total = static_cast<long long>(B) * np * K;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(e % K);
    const long long r = e / K;
    const int patch = static_cast<int>(r % np);
    const int b = static_cast<int>(r / np);
    const int c = k / (p * p), kh = (k / p) % p, kw = k % p;
    const int y = (patch / g) * p + kh, x = (patch % g) * p + kw;
    out[e] = __float2bfloat16_rn(img[((static_cast<long long>(b) * C + c) * I + y) * I + x]);
  }
}

// The same for 16 x 16 patches, one patch row per thread: 16 consecutive pixels of one
// channel (64 bytes of the image row, four float4 loads) become 16 consecutive bf16 of the
// patch's column vector (two 16-byte stores); the index arithmetic runs once per 16
// elements in 32-bit.  Thread t = ((b np + patch) C + c) 16 + kh.
__global__ void im2col_patches16_kernel(const float* __restrict__ img, __nv_bfloat16* __restrict__ out, int B,
                                        int C, int I) {
  constexpr int p = 16;
  const int g = I / p, np = g * g;
  const int total = B * np * C * p;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
    const int kh = t % p;
    const int c = (t / p) % C;
    const int bp = t / (p * C);  // b np + patch
    const int patch = bp % np, b = bp / np;
    const int y = (patch / g) * p + kh, x0 = (patch % g) * p;
    const float4* src = reinterpret_cast<const float4*>(img + ((static_cast<long long>(b) * C + c) * I + y) * I + x0);
    uint32_t w[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = src[q];
      w[2 * q] = pack_bf16x2(v.x, v.y);
      w[2 * q + 1] = pack_bf16x2(v.z, v.w);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(bp) * (C * p * p) + c * p * p + kh * p);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

template <int VPL>
__global__ void __launch_bounds__(kWarps * 32)
    vit_assemble_fwd_kernel(const __nv_bfloat16* __restrict__ conv, const float* __restrict__ cls,
                            const float* __restrict__ pos, const float* __restrict__ gamma,
                            const float* __restrict__ beta, float eps, int B, int S, float* __restrict__ out) {
  constexpr int H = VPL * 128;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= B * S) return;
  const int b = row / S, s = row % S;
  float4 v[VPL];
  const float4* p4 = reinterpret_cast<const float4*>(pos + static_cast<long long>(s) * H);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    float4 a;
    if (s == 0) {
      a = __ldg(reinterpret_cast<const float4*>(cls) + c);
    } else {
      const uint2 q = *reinterpret_cast<const uint2*>(conv + (static_cast<long long>(b) * (S - 1) + s - 1) * H + 4 * c);
      const float2 lo = unpack_bf16x2(q.x), hi = unpack_bf16x2(q.y);
      a = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    v[i] = f4add(a, __ldg(p4 + c));
  }
  float mean, rstd;
  row_stats<VPL>(v, mean, rstd, eps);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  float4* o4 = reinterpret_cast<float4*>(out + static_cast<long long>(row) * H);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    const float4 g = __ldg(g4 + c), bb = __ldg(b4 + c);
    o4[c] = make_float4((v[i].x - mean) * rstd * g.x + bb.x, (v[i].y - mean) * rstd * g.y + bb.y,
                        (v[i].z - mean) * rstd * g.z + bb.z, (v[i].w - mean) * rstd * g.w + bb.w);
  }
}

// grid = S (one CTA per token position), loops over the batch.
// grid = S (one CTA per token position), 8 warps; the batch rows of the position are taken 8
// at a time, one per warp, as in bert_embed_bwd_kernel: per-row gradients go to shared
// memory, each thread sums its columns over the rows in registers (no shared-memory atomics).
template <int VPL>
__global__ void __launch_bounds__(kWarps * 32)
    vit_assemble_bwd_kernel(const __nv_bfloat16* __restrict__ conv, const float* __restrict__ cls,
                            const float* __restrict__ pos, const float* __restrict__ gamma, float eps, int B, int S,
                            const float* __restrict__ dx2, const float* __restrict__ dx1,
                            __nv_bfloat16* __restrict__ dconv, float* __restrict__ dcls, float* __restrict__ dpos,
                            float* __restrict__ dgamma, float* __restrict__ dbeta) {
  constexpr int H = VPL * 128;
  constexpr int NT = kWarps * 32;
  constexpr int J = (H + NT - 1) / NT;
  extern __shared__ float4 sbuf4[];  // [3][kWarps][H / 4]: dv, dy * x-hat, dy
  float* sbuf = reinterpret_cast<float*>(sbuf4);
  const int s = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* p4 = reinterpret_cast<const float4*>(pos + static_cast<long long>(s) * H);
  float apos[J], ag[J], ab[J];
#pragma unroll
  for (int j = 0; j < J; ++j) apos[j] = ag[j] = ab[j] = 0.f;
  for (int b0 = 0; b0 < B; b0 += kWarps) {
    const int b = b0 + warp;
    if (b < B) {
      const long long row = static_cast<long long>(b) * S + s;
      float4 v[VPL], dy[VPL];
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int c = lane + 32 * i;
        float4 a;
        if (s == 0) {
          a = __ldg(reinterpret_cast<const float4*>(cls) + c);
        } else {
          const uint2 q =
              *reinterpret_cast<const uint2*>(conv + (static_cast<long long>(b) * (S - 1) + s - 1) * H + 4 * c);
          const float2 lo = unpack_bf16x2(q.x), hi = unpack_bf16x2(q.y);
          a = make_float4(lo.x, lo.y, hi.x, hi.y);
        }
        v[i] = f4add(a, __ldg(p4 + c));
        dy[i] = reinterpret_cast<const float4*>(dx2 + row * H)[c];
        if (dx1) dy[i] = f4add(dy[i], reinterpret_cast<const float4*>(dx1 + row * H)[c]);
      }
      float mean, rstd;
      row_stats<VPL>(v, mean, rstd, eps);
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const float4 g = __ldg(g4 + lane + 32 * i);
        v[i] = make_float4((v[i].x - mean) * rstd, (v[i].y - mean) * rstd, (v[i].z - mean) * rstd,
                           (v[i].w - mean) * rstd);
        s1 += dy[i].x * g.x + dy[i].y * g.y + dy[i].z * g.z + dy[i].w * g.w;
        s2 += dy[i].x * g.x * v[i].x + dy[i].y * g.y * v[i].y + dy[i].z * g.z * v[i].z + dy[i].w * g.w * v[i].w;
      }
      const float m1 = warp_sum(s1) * (1.0f / H), m2 = warp_sum(s2) * (1.0f / H);
      float4* r_dv = sbuf4 + (0 * kWarps + warp) * (H / 4);
      float4* r_dx = sbuf4 + (1 * kWarps + warp) * (H / 4);
      float4* r_dy = sbuf4 + (2 * kWarps + warp) * (H / 4);
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int c4 = lane + 32 * i;
        const float4 g = __ldg(g4 + c4);
        const float4 dv = make_float4(rstd * (dy[i].x * g.x - m1 - v[i].x * m2), rstd * (dy[i].y * g.y - m1 - v[i].y * m2),
                                      rstd * (dy[i].z * g.z - m1 - v[i].z * m2), rstd * (dy[i].w * g.w - m1 - v[i].w * m2));
        if (s > 0) {
          *reinterpret_cast<uint2*>(dconv + (static_cast<long long>(b) * (S - 1) + s - 1) * H + 4 * c4) =
              make_uint2(pack_bf16x2(dv.x, dv.y), pack_bf16x2(dv.z, dv.w));
        }
        r_dv[c4] = dv;
        r_dx[c4] = make_float4(dy[i].x * v[i].x, dy[i].y * v[i].y, dy[i].z * v[i].z, dy[i].w * v[i].w);
        r_dy[c4] = dy[i];
      }
    }
    __syncthreads();
    const int nr = min(kWarps, B - b0);
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = threadIdx.x + NT * j;
      if (c < H) {
        for (int r = 0; r < nr; ++r) {
          apos[j] += sbuf[(0 * kWarps + r) * H + c];
          ag[j] += sbuf[(1 * kWarps + r) * H + c];
          ab[j] += sbuf[(2 * kWarps + r) * H + c];
        }
      }
    }
    __syncthreads();  // the buffers are rewritten by the next chunk
  }
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = threadIdx.x + NT * j;
    if (c >= H) continue;
    dpos[static_cast<long long>(s) * H + c] += apos[j];
    if (s == 0) dcls[c] += apos[j];
    atomicAdd(dgamma + c, ag[j]);
    atomicAdd(dbeta + c, ab[j]);
  }
}

// ------------------------------------------------------------------ head
// pooled[b, :] : mode 0 mean over S of (y2 + y1); mode 1 row 0 of (y2 + y1);
//                mode 2 row 0 of concat [y1, y2] (width 2H); y1 may be null (single stream).
__global__ void head_pool_kernel(const float* __restrict__ y2, const float* __restrict__ y1, int B, int S, int H,
                                 int mode, float* __restrict__ pooled) {
  const int b = blockIdx.y;
  const int W = mode == 2 ? 2 * H : H;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= W) return;
  const long long base = static_cast<long long>(b) * S * H;
  float acc = 0.f;
  if (mode == 0) {
    for (int s = 0; s < S; ++s) {
      acc += y2[base + static_cast<long long>(s) * H + c];
      if (y1) acc += y1[base + static_cast<long long>(s) * H + c];
    }
    acc *= 1.0f / S;
  } else if (mode == 1) {
    acc = y2[base + c] + (y1 ? y1[base + c] : 0.f);
  } else {
    acc = c < H ? y1[base + c] : y2[base + c - H];
  }
  pooled[static_cast<long long>(b) * W + c] = acc;
}

// The classifier head runs as small batched kernels, each over the whole micro-batch:
//   head_ln_fwd_kernel   one CTA per sample: LayerNorm statistics, hb = bf16(LN(pooled))
//   head_logits_kernel   (class block, sample block): logits = bf16(hb W^T + b)
//   head_ce_kernel       one CTA per sample: softmax cross-entropy, loss, dlogits
//   head_dgrad_kernel    (column block, sample block, class chunk): dyp = bf16(dlogits) W
//   head_ln_bwd_kernel   one CTA per sample: dpooled, dgamma, dbeta
//   head_wgrad_kernel    dW, db
// (one CTA per sample for everything took 731 us for 16 ImageNet samples of ViT-L: its
// class loops ran on 16 SMs).

// Block reduction of one float over the CTA (all threads get the result); red: 33 floats.
__device__ __forceinline__ float head_block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float u = lane < nw ? red[lane] : 0.f;
    u = warp_sum(u);
    if (lane == 0) red[32] = u;
  }
  __syncthreads();
  return red[32];
}
__device__ __forceinline__ float head_block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float u = lane < nw ? red[lane] : -INFINITY;
    u = warp_max(u);
    if (lane == 0) red[32] = u;
  }
  __syncthreads();
  return red[32];
}

// hb[b, :] = bf16(LN(pooled[b, :]) gamma + beta); stats[b] = (mean, rstd).  One CTA per sample.
__global__ void head_ln_fwd_kernel(const float* __restrict__ pooled, int W, const float* __restrict__ gamma,
                                   const float* __restrict__ beta, float eps, __nv_bfloat16* __restrict__ hb,
                                   float* __restrict__ stats) {
  __shared__ float red[33];
  const int b = blockIdx.x;
  const float* x = pooled + static_cast<long long>(b) * W;
  float s = 0.f;
  for (int i = threadIdx.x; i < W; i += blockDim.x) s += x[i];
  const float mean = head_block_sum(s, red) / W;
  float ss = 0.f;
  for (int i = threadIdx.x; i < W; i += blockDim.x) {
    const float d = x[i] - mean;
    ss += d * d;
  }
  const float rstd = rsqrtf(head_block_sum(ss, red) / W + eps);
  if (threadIdx.x == 0) {
    stats[2 * b] = mean;
    stats[2 * b + 1] = rstd;
  }
  for (int i = threadIdx.x; i < W; i += blockDim.x)
    hb[static_cast<long long>(b) * W + i] = __float2bfloat16_rn((x[i] - mean) * rstd * gamma[i] + beta[i]);
}

// logits[b, c] = bf16(sum_i hb[b, i] W[c, i] + bias[c]).  Block (x, y): classes 8 x .. 8 x + 7
// (one per warp), samples 16 y .. 16 y + 15, whose hb rows sit in shared memory (bf16).  A warp
// reads a class row of W once (coalesced) for its 16 samples; lane l takes elements
// l, l + 32, ... of the row.
constexpr int kHeadLgClasses = 8;
constexpr int kHeadLgSamples = 16;
__global__ void __launch_bounds__(256) head_logits_kernel(const __nv_bfloat16* __restrict__ hb,
                                                          const __nv_bfloat16* __restrict__ wb,
                                                          const __nv_bfloat16* __restrict__ bb, int B, int C, int W,
                                                          float* __restrict__ logits) {
  extern __shared__ __nv_bfloat16 shb[];  // [kHeadLgSamples][W]
  const int b0 = blockIdx.y * kHeadLgSamples;
  const int nb = min(kHeadLgSamples, B - b0);
  for (int e = threadIdx.x; e < kHeadLgSamples * W; e += blockDim.x) {
    const int sb = e / W, i = e % W;
    shb[e] = sb < nb ? hb[static_cast<long long>(b0 + sb) * W + i] : __float2bfloat16_rn(0.f);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int cc = 0; cc < kHeadLgClasses / 8; ++cc) {
    const int c = blockIdx.x * kHeadLgClasses + warp * (kHeadLgClasses / 8) + cc;
    if (c >= C) break;
    const __nv_bfloat16* wr = wb + static_cast<long long>(c) * W;
    float acc[kHeadLgSamples];
#pragma unroll
    for (int k = 0; k < kHeadLgSamples; ++k) acc[k] = 0.f;
    for (int i = lane; i < W; i += 32) {
      const float w = __bfloat162float(wr[i]);
#pragma unroll
      for (int k = 0; k < kHeadLgSamples; ++k) acc[k] = fmaf(__bfloat162float(shb[k * W + i]), w, acc[k]);
    }
    const float bias = __bfloat162float(bb[c]);
#pragma unroll
    for (int k = 0; k < kHeadLgSamples; ++k) {
      const float v = warp_sum(acc[k]);
      if (lane == 0 && k < nb) logits[static_cast<long long>(b0 + k) * C + c] = bf16r(v + bias);
    }
  }
}

// Softmax cross-entropy of one sample per CTA: loss[b] = lse - logit[label]; with want_grad
// dlogits[b, c] = (softmax - onehot) grad_scale / B.
__global__ void head_ce_kernel(const float* __restrict__ logits, int C, const int64_t* __restrict__ labels,
                               float grad_scale, int B, float* __restrict__ loss_out, float* __restrict__ dlogits,
                               int want_grad, int* __restrict__ status) {
  __shared__ float red[33];
  const int b = blockIdx.x;
  const float* lg = logits + static_cast<long long>(b) * C;
  float mx = -INFINITY;
  for (int c = threadIdx.x; c < C; c += blockDim.x) mx = fmaxf(mx, lg[c]);
  mx = head_block_max(mx, red);
  float se = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) se += expf(lg[c] - mx);
  const float lse = mx + logf(head_block_sum(se, red));
  long long lab = labels ? labels[b] : 0;
  if (lab < 0 || lab >= C) {
    if (threadIdx.x == 0 && status) atomicOr(status, kStatusBadShape);
    lab = 0;
  }
  if (threadIdx.x == 0 && loss_out) loss_out[b] = lse - lg[lab];
  if (!want_grad) return;
  const float sc = grad_scale / B;
  for (int c = threadIdx.x; c < C; c += blockDim.x)
    dlogits[static_cast<long long>(b) * C + c] = (expf(lg[c] - lse) - (c == lab ? 1.f : 0.f)) * sc;
}

// dyp[b, i] += sum over a chunk of classes c of bf16(dlogits[b, c]) W[c, i]: the input
// gradient of the head's linear layer, the LayerNorm backward still to come.  Block (x, y, z):
// columns 128 x .. 128 x + 127 (one per thread), samples 16 y .. 16 y + 15, classes
// z cpb .. z cpb + cpb - 1 (their logit gradients staged in shared memory, read as
// broadcasts); partial sums of the class chunks meet in dyp with atomics.  Replaces a loop
// over all classes per column and sample in one CTA per sample (731 us for 16 ImageNet
// samples of ViT-L).
constexpr int kHeadDgSamples = 16;
__global__ void __launch_bounds__(128) head_dgrad_kernel(const float* __restrict__ dlogits,
                                                         const __nv_bfloat16* __restrict__ wb, int B, int C, int W,
                                                         int cpb, float* __restrict__ dyp) {
  extern __shared__ float sdl[];  // [kHeadDgSamples][cpb]
  const int i = blockIdx.x * 128 + threadIdx.x;
  const int b0 = blockIdx.y * kHeadDgSamples;
  const int c0 = blockIdx.z * cpb;
  const int c1 = min(C, c0 + cpb);
  const int nb = min(kHeadDgSamples, B - b0);
  for (int e = threadIdx.x; e < kHeadDgSamples * cpb; e += blockDim.x) {
    const int sb = e / cpb, sc = e % cpb;
    sdl[e] = (sb < nb && c0 + sc < C) ? bf16r(dlogits[static_cast<long long>(b0 + sb) * C + c0 + sc]) : 0.f;
  }
  __syncthreads();
  if (i >= W || c0 >= C) return;
  float acc[kHeadDgSamples];
#pragma unroll
  for (int k = 0; k < kHeadDgSamples; ++k) acc[k] = 0.f;
#pragma unroll 4
  for (int c = c0; c < c1; ++c) {
    const float w = __bfloat162float(wb[static_cast<long long>(c) * W + i]);
    const float* d = sdl + (c - c0);
#pragma unroll
    for (int k = 0; k < kHeadDgSamples; ++k) acc[k] = fmaf(d[k * cpb], w, acc[k]);
  }
#pragma unroll
  for (int k = 0; k < kHeadDgSamples; ++k)
    if (k < nb) atomicAdd(dyp + static_cast<long long>(b0 + k) * W + i, acc[k]);
}

// LayerNorm backward of the head, one CTA per sample: dpooled from dyp (the gradient of the
// LayerNorm output), and dgamma / dbeta += their per-sample terms.
__global__ void head_ln_bwd_kernel(const float* __restrict__ pooled, const float* __restrict__ stats, int W,
                                   const float* __restrict__ gamma, const float* __restrict__ dyp,
                                   float* __restrict__ dpooled, float* __restrict__ dgamma,
                                   float* __restrict__ dbeta) {
  __shared__ float red[66];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  const float mean = stats[2 * b], rstd = stats[2 * b + 1];
  const float* x = pooled + static_cast<long long>(b) * W;
  const float* dy = dyp + static_cast<long long>(b) * W;
  float a1 = 0.f, a2 = 0.f;
  for (int i = tid; i < W; i += nt) {
    const float xh = (x[i] - mean) * rstd;
    const float d = dy[i];
    const float g = d * gamma[i];
    a1 += g;
    a2 += g * xh;
    atomicAdd(dgamma + i, d * xh);
    atomicAdd(dbeta + i, d);
  }
  a1 = warp_sum(a1);
  a2 = warp_sum(a2);
  if (lane == 0) {
    red[warp] = a1;
    red[32 + warp] = a2;
  }
  __syncthreads();
  if (warp == 0) {
    float u = lane < nw ? red[lane] : 0.f, v = lane < nw ? red[32 + lane] : 0.f;
    u = warp_sum(u);
    v = warp_sum(v);
    if (lane == 0) {
      red[64] = u / W;
      red[65] = v / W;
    }
  }
  __syncthreads();
  const float m1 = red[64], m2 = red[65];
  for (int i = tid; i < W; i += nt) {
    const float xh = (x[i] - mean) * rstd;
    dpooled[static_cast<long long>(b) * W + i] = rstd * (dy[i] * gamma[i] - m1 - xh * m2);
  }
}

// dW[c, i] += sum_b bf16(dlogits[b, c]) * hb[b, i];  db[c] += sum_b dlogits[b, c]
__global__ void head_wgrad_kernel(const float* __restrict__ dlogits, const __nv_bfloat16* __restrict__ hb, int B,
                                  int C, int W, float* __restrict__ dW, float* __restrict__ db) {
  const long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (e >= static_cast<long long>(C) * W) return;
  const int c = static_cast<int>(e / W), i = static_cast<int>(e % W);
  float acc = 0.f, accb = 0.f;
  for (int b = 0; b < B; ++b) {
    const float d = dlogits[static_cast<long long>(b) * C + c];
    acc += bf16r(d) * __bfloat162float(hb[static_cast<long long>(b) * W + i]);
    accb += d;
  }
  dW[e] += acc;
  if (i == 0) db[c] += accb;
}

// dY[b, s, :] from dpooled[b, :]: mode 0 -> dpooled / S on every row, mode 1 -> row 0 only,
// mode 2 (concat) -> dy1 = first half, dy2 = second half, row 0 only.
__global__ void head_spread_kernel(const float* __restrict__ dpooled, int B, int S, int H, int mode,
                                   float* __restrict__ dy2, float* __restrict__ dy1) {
  const long long n4 = static_cast<long long>(B) * S * H / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = i * 4;
    const int c = static_cast<int>(e % H);
    const long long r = e / H;
    const int s = static_cast<int>(r % S), b = static_cast<int>(r / S);
    float4 v2 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v2;
    if (mode == 0) {
      const float4 p = *reinterpret_cast<const float4*>(dpooled + static_cast<long long>(b) * H + c);
      const float inv = 1.0f / S;
      v2 = make_float4(p.x * inv, p.y * inv, p.z * inv, p.w * inv);
      v1 = v2;
    } else if (s == 0) {
      if (mode == 1) {
        v2 = *reinterpret_cast<const float4*>(dpooled + static_cast<long long>(b) * H + c);
        v1 = v2;
      } else {
        v1 = *reinterpret_cast<const float4*>(dpooled + static_cast<long long>(b) * 2 * H + c);
        v2 = *reinterpret_cast<const float4*>(dpooled + static_cast<long long>(b) * 2 * H + H + c);
      }
    }
    reinterpret_cast<float4*>(dy2)[i] = v2;
    if (dy1) reinterpret_cast<float4*>(dy1)[i] = v1;
  }
}

// ------------------------------------------------------------------ host side
namespace {
template <typename F>
void vpl_dispatch(int H, F&& f) {
  REVPP_CHECK(H % 128 == 0 && H >= 128 && H <= 2048, "width must be a multiple of 128 in [128, 2048], got ", H);
  switch (H / 128) {
    case 1: f(std::integral_constant<int, 1>{}); break;
    case 2: f(std::integral_constant<int, 2>{}); break;
    case 4: f(std::integral_constant<int, 4>{}); break;
    case 6: f(std::integral_constant<int, 6>{}); break;
    case 8: f(std::integral_constant<int, 8>{}); break;
    case 12: f(std::integral_constant<int, 12>{}); break;
    case 16: f(std::integral_constant<int, 16>{}); break;
    default: REVPP_CHECK(false, "unsupported width ", H);
  }
}
int grid1d(long long n, int threads) {
  return static_cast<int>(std::max<long long>(1, std::min<long long>((n + threads - 1) / threads, 16LL * num_sms())));
}
}  // namespace

void bert_embed_fwd(const torch::Tensor& ids, const torch::Tensor& tt, const torch::Tensor& word,
                    const torch::Tensor& pos, const torch::Tensor& type, const torch::Tensor& gamma,
                    const torch::Tensor& beta, double eps, torch::Tensor out) {
  REVPP_CHECK(ids.scalar_type() == at::kLong && tt.scalar_type() == at::kLong, "ids must be int64");
  REVPP_CHECK(ids.is_contiguous() && tt.is_contiguous() && ids.sizes() == tt.sizes() && ids.dim() == 2, "ids [B, S]");
  check_cuda_f32(out, "out");
  const int B = static_cast<int>(ids.size(0)), S = static_cast<int>(ids.size(1));
  const int H = static_cast<int>(word.size(1));
  REVPP_CHECK(pos.size(0) >= S, "sequence longer than the position table");
  c10::cuda::CUDAGuard guard(ids.device());
  const int M = B * S;
  vpl_dispatch(H, [&](auto v) {
    bert_embed_fwd_kernel<decltype(v)::value><<<(M + kWarps - 1) / kWarps, kWarps * 32, 0, cur_stream()>>>(
        ids.data_ptr<int64_t>(), tt.data_ptr<int64_t>(), word.data_ptr<float>(), pos.data_ptr<float>(),
        type.data_ptr<float>(), gamma.data_ptr<float>(), beta.data_ptr<float>(), static_cast<float>(eps), M, S,
        static_cast<int>(word.size(0)), static_cast<int>(type.size(0)), out.data_ptr<float>(), status_device_ptr());
  });
  REVPP_CHECK_LAUNCH();
}

void bert_embed_bwd(const torch::Tensor& ids, const torch::Tensor& tt, const torch::Tensor& word,
                    const torch::Tensor& pos, const torch::Tensor& type, const torch::Tensor& gamma, double eps,
                    const torch::Tensor& dx2, const c10::optional<torch::Tensor>& dx1, torch::Tensor dword,
                    torch::Tensor dpos, torch::Tensor dtype, torch::Tensor dgamma, torch::Tensor dbeta) {
  const int B = static_cast<int>(ids.size(0)), S = static_cast<int>(ids.size(1));
  const int H = static_cast<int>(word.size(1));
  const int T = static_cast<int>(type.size(0));
  check_cuda_f32(dx2, "dx2");
  REVPP_CHECK(dx2.is_contiguous() && dx2.numel() == static_cast<long long>(B) * S * H, "dx2 [B, S, H]");
  const float* d1 = nullptr;
  if (dx1.has_value() && dx1->defined()) {
    REVPP_CHECK(dx1->is_contiguous() && dx1->numel() == dx2.numel(), "dx1 [B, S, H]");
    d1 = dx1->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(ids.device());
  REVPP_CHECK(T <= kEmbedMaxTypes, "type vocabulary above ", kEmbedMaxTypes, " types");
  const int smem = 3 * kWarps * H * 4;
  vpl_dispatch(H, [&](auto v) {
    auto k = bert_embed_bwd_kernel<decltype(v)::value>;
    if (smem > 48 * 1024) REVPP_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    k<<<S, kWarps * 32, smem, cur_stream()>>>(
        ids.data_ptr<int64_t>(), tt.data_ptr<int64_t>(), word.data_ptr<float>(), pos.data_ptr<float>(),
        type.data_ptr<float>(), gamma.data_ptr<float>(), static_cast<float>(eps), B, S, static_cast<int>(word.size(0)),
        T, dx2.data_ptr<float>(), d1, dword.data_ptr<float>(), dpos.data_ptr<float>(), dtype.data_ptr<float>(),
        dgamma.data_ptr<float>(), dbeta.data_ptr<float>());
  });
  REVPP_CHECK_LAUNCH();
}

void im2col_patches(const torch::Tensor& img, int64_t patch, torch::Tensor out) {
  check_cuda_f32(img, "img");
  check_cuda_bf16(out, "out");
  REVPP_CHECK(img.is_contiguous() && img.dim() == 4 && img.size(2) == img.size(3), "img [B, C, I, I]");
  const int B = static_cast<int>(img.size(0)), C = static_cast<int>(img.size(1)), I = static_cast<int>(img.size(2));
  const int p = static_cast<int>(patch);
  REVPP_CHECK(I % p == 0, "image size must be a multiple of the patch size");
  const long long n = static_cast<long long>(B) * (I / p) * (I / p) * C * p * p;
  REVPP_CHECK(out.numel() >= n, "patch buffer too small");
  c10::cuda::CUDAGuard guard(img.device());
  const bool vec16 = p == 16 && I % 16 == 0 && (reinterpret_cast<uintptr_t>(img.data_ptr()) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0 &&
                     static_cast<long long>(B) * C * I * I < (1LL << 31);
  if (vec16) {
    const long long rows = static_cast<long long>(B) * (I / 16) * (I / 16) * C * 16;
    im2col_patches16_kernel<<<grid1d(rows, 256), 256, 0, cur_stream()>>>(
        img.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), B, C, I);
  } else {
    im2col_patches_kernel<<<grid1d(n, 256), 256, 0, cur_stream()>>>(img.data_ptr<float>(),
                                                                      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                                      B, C, I, p);
  }
  REVPP_CHECK_LAUNCH();
}

void vit_assemble_fwd(const torch::Tensor& conv, const torch::Tensor& cls, const torch::Tensor& pos,
                      const torch::Tensor& gamma, const torch::Tensor& beta, double eps, int64_t B, int64_t S,
                      torch::Tensor out) {
  check_cuda_bf16(conv, "conv");
  const int H = static_cast<int>(gamma.numel());
  c10::cuda::CUDAGuard guard(conv.device());
  const int M = static_cast<int>(B * S);
  vpl_dispatch(H, [&](auto v) {
    vit_assemble_fwd_kernel<decltype(v)::value><<<(M + kWarps - 1) / kWarps, kWarps * 32, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(conv.data_ptr()), cls.data_ptr<float>(), pos.data_ptr<float>(),
        gamma.data_ptr<float>(), beta.data_ptr<float>(), static_cast<float>(eps), static_cast<int>(B),
        static_cast<int>(S), out.data_ptr<float>());
  });
  REVPP_CHECK_LAUNCH();
}

void vit_assemble_bwd(const torch::Tensor& conv, const torch::Tensor& cls, const torch::Tensor& pos,
                      const torch::Tensor& gamma, double eps, int64_t B, int64_t S, const torch::Tensor& dx2,
                      const c10::optional<torch::Tensor>& dx1, torch::Tensor dconv, torch::Tensor dcls,
                      torch::Tensor dpos, torch::Tensor dgamma, torch::Tensor dbeta) {
  const int H = static_cast<int>(gamma.numel());
  c10::cuda::CUDAGuard guard(conv.device());
  const float* d1 = (dx1.has_value() && dx1->defined()) ? dx1->data_ptr<float>() : nullptr;
  const int smem = 3 * kWarps * H * 4;
  vpl_dispatch(H, [&](auto v) {
    auto k = vit_assemble_bwd_kernel<decltype(v)::value>;
    if (smem > 48 * 1024) REVPP_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    k<<<static_cast<unsigned>(S), kWarps * 32, smem, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(conv.data_ptr()), cls.data_ptr<float>(), pos.data_ptr<float>(),
        gamma.data_ptr<float>(), static_cast<float>(eps), static_cast<int>(B), static_cast<int>(S),
        dx2.data_ptr<float>(), d1, reinterpret_cast<__nv_bfloat16*>(dconv.data_ptr()), dcls.data_ptr<float>(),
        dpos.data_ptr<float>(), dgamma.data_ptr<float>(), dbeta.data_ptr<float>());
  });
  REVPP_CHECK_LAUNCH();
}

// mode: 0 mean-pool of y2 + y1, 1 CLS row of y2 + y1, 2 CLS row of concat [y1, y2].
// Returns nothing; fills logits [B, C], loss [B]; with want_grad also the parameter
// gradients and dy2 / dy1 ([B, S, H]).
void head_fwd_bwd(const torch::Tensor& y2, const c10::optional<torch::Tensor>& y1, int64_t mode,
                  const torch::Tensor& gamma, const torch::Tensor& beta, double eps, const torch::Tensor& wb,
                  const torch::Tensor& bb, const c10::optional<torch::Tensor>& labels, double grad_scale,
                  torch::Tensor pooled, torch::Tensor logits, torch::Tensor loss, bool want_grad,
                  const c10::optional<torch::Tensor>& dlogits, const c10::optional<torch::Tensor>& hb,
                  const c10::optional<torch::Tensor>& dpooled, const c10::optional<torch::Tensor>& dW,
                  const c10::optional<torch::Tensor>& db, const c10::optional<torch::Tensor>& dgamma,
                  const c10::optional<torch::Tensor>& dbeta, const c10::optional<torch::Tensor>& dy2,
                  const c10::optional<torch::Tensor>& dy1) {
  check_cuda_f32(y2, "y2");
  const int B = static_cast<int>(y2.size(0)), S = static_cast<int>(y2.size(1)), H = static_cast<int>(y2.size(2));
  const int W = mode == 2 ? 2 * H : H;
  const int C = static_cast<int>(wb.size(0));
  REVPP_CHECK(wb.size(1) == W && gamma.numel() == W, "head width mismatch");
  const float* y1p = (y1.has_value() && y1->defined()) ? y1->data_ptr<float>() : nullptr;
  REVPP_CHECK(mode != 2 || y1p != nullptr, "concat pooling needs both streams");
  c10::cuda::CUDAGuard guard(y2.device());
  cudaStream_t st = cur_stream();
  {
    dim3 grid((W + 255) / 256, B);
    head_pool_kernel<<<grid, 256, 0, st>>>(y2.data_ptr<float>(), y1p, B, S, H, static_cast<int>(mode),
                                            pooled.data_ptr<float>());
    REVPP_CHECK_LAUNCH();
  }
  const int64_t* lab = (labels.has_value() && labels->defined()) ? labels->data_ptr<int64_t>() : nullptr;
  torch::Tensor stats = torch::empty({B, 2}, y2.options());
  torch::Tensor hbt = (want_grad && hb.has_value() && hb->defined())
                          ? *hb
                          : torch::empty({B, W}, y2.options().dtype(at::kBFloat16));
  auto* hbp = reinterpret_cast<__nv_bfloat16*>(hbt.data_ptr());
  head_ln_fwd_kernel<<<B, 256, 0, st>>>(pooled.data_ptr<float>(), W, gamma.data_ptr<float>(),
                                         beta.data_ptr<float>(), static_cast<float>(eps), hbp,
                                         stats.data_ptr<float>());
  REVPP_CHECK_LAUNCH();
  {
    const int lsmem = kHeadLgSamples * W * 2;
    static int configured_for = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (lsmem > 48 * 1024 && configured_for != dev) {
      REVPP_CUDA_CHECK(cudaFuncSetAttribute(head_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            kHeadLgSamples * 4096 * 2));
      configured_for = dev;
    }
    REVPP_CHECK(W <= 4096, "head: width above 4096");
    dim3 grid((C + kHeadLgClasses - 1) / kHeadLgClasses, (B + kHeadLgSamples - 1) / kHeadLgSamples);
    head_logits_kernel<<<grid, 256, lsmem, st>>>(hbp, reinterpret_cast<const __nv_bfloat16*>(wb.data_ptr()),
                                                 reinterpret_cast<const __nv_bfloat16*>(bb.data_ptr()), B, C, W,
                                                 logits.data_ptr<float>());
    REVPP_CHECK_LAUNCH();
  }
  head_ce_kernel<<<B, 256, 0, st>>>(logits.data_ptr<float>(), C, lab, static_cast<float>(grad_scale), B,
                                     loss.data_ptr<float>(), want_grad ? dlogits->data_ptr<float>() : nullptr,
                                     want_grad ? 1 : 0, status_device_ptr());
  REVPP_CHECK_LAUNCH();
  if (!want_grad) return;
  {
    // input gradient: dyp = bf16(dlogits) W over class chunks, then the LayerNorm backward
    torch::Tensor dyp = torch::zeros({B, W}, y2.options());
    const int gx = (W + 127) / 128, gy = (B + kHeadDgSamples - 1) / kHeadDgSamples;
    const int want = std::max(1, (num_sms() + gx * gy - 1) / (gx * gy));
    const int cpb = std::max(16, (C + want - 1) / want);
    const int gz = (C + cpb - 1) / cpb;
    const int dsmem = kHeadDgSamples * cpb * 4;
    REVPP_CHECK(dsmem <= 48 * 1024, "head: class chunk too large");
    head_dgrad_kernel<<<dim3(gx, gy, gz), 128, dsmem, st>>>(
        dlogits->data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(wb.data_ptr()), B, C, W, cpb,
        dyp.data_ptr<float>());
    REVPP_CHECK_LAUNCH();
    head_ln_bwd_kernel<<<B, 256, 0, st>>>(pooled.data_ptr<float>(), stats.data_ptr<float>(), W,
                                           gamma.data_ptr<float>(), dyp.data_ptr<float>(),
                                           dpooled->data_ptr<float>(), dgamma->data_ptr<float>(),
                                           dbeta->data_ptr<float>());
    REVPP_CHECK_LAUNCH();
  }
  {
    const long long n = static_cast<long long>(C) * W;
    head_wgrad_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(
        dlogits->data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(hb->data_ptr()), B, C, W,
        dW->data_ptr<float>(), db->data_ptr<float>());
    REVPP_CHECK_LAUNCH();
  }
  {
    const long long n4 = static_cast<long long>(B) * S * H / 4;
    float* d1p = (dy1.has_value() && dy1->defined()) ? dy1->data_ptr<float>() : nullptr;
    head_spread_kernel<<<grid1d(n4, 256), 256, 0, st>>>(dpooled->data_ptr<float>(), B, S, H, static_cast<int>(mode),
                                                        dy2->data_ptr<float>(), d1p);
    REVPP_CHECK_LAUNCH();
  }
}

}  // namespace revpp
