// Flash attention forward / backward, head dim 64, no mask (the reference runs
// nn.MultiheadAttention without a mask, BERT/models/bert_blocks.py:50-63), keys
// past the sequence end (tiles that straddle S) are masked.
//
// Input  qkv [B*S, 3H] bf16, packed as nn.MultiheadAttention's in_proj output:
//        q = cols [0, H), k = [H, 2H), v = [2H, 3H); head h uses 64 columns h*64.
// Output o   [B*S, H]  bf16 (heads concatenated, the layout out_proj reads),
//        lse [B, heads, S] fp32 natural-log row sums for the backward.
// Backward writes dqkv [B*S, 3H] bf16 in the same packed layout.
//
// The softmax probabilities are never materialised (the reference's math path
// keeps [B*heads, S, S] per block).  Warp-level mma.sync m16n8k16 tiles; the
// tcgen05 path for this op lives in attention_tc.cu.
#include "common.cuh"
#include "host.h"

namespace revpp {

namespace {

constexpr int kD = 64;        // head dim
constexpr int kTileQ = 64;    // query rows per CTA (16 per warp)
constexpr int kTileK = 64;    // keys per tile
constexpr int kWarps = 4;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = smem_u32(smem);
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Row r of a [rows x 64] bf16 tile, 16-byte chunk c, XOR-swizzled to avoid
// ldmatrix bank conflicts.
__device__ __forceinline__ int swz(int r, int c) { return r * 64 + ((c ^ (r & 7)) << 3); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Load a [64 x 64] bf16 tile (rows row0.., 64 columns at col0) into swizzled smem.
// Rows >= row_end are zero-filled.
__device__ __forceinline__ void load_tile(__nv_bfloat16* s, const __nv_bfloat16* g, long long ld, int row0,
                                          int row_end, int col0, int tid, int nthreads) {
  for (int i = tid; i < 64 * 8; i += nthreads) {
    const int r = i >> 3, c = i & 7;
    const int gr = row0 + r;
    const bool ok = gr < row_end;
    const __nv_bfloat16* src = g + static_cast<long long>(ok ? gr : row0) * ld + col0 + c * 8;
    cp_async16(s + swz(r, c), src, ok);
  }
}

// A fragment (16 rows x 16 k) from a swizzled row-major tile: rows r0.., k chunk kk (16 wide).
__device__ __forceinline__ void lda_frag(uint32_t (&a)[4], const __nv_bfloat16* s, int r0, int kk, int lane) {
  const int r = r0 + (lane & 15);
  const int c = kk * 2 + (lane >> 4);
  ldsm_x4(a, s + swz(r, c));
}
// B fragments for two n8 tiles (n rows n0..n0+15 of a [n x k] row-major tile), k chunk kk.
// Returns {b0(n0), b1(n0), b0(n0+8), b1(n0+8)}.
__device__ __forceinline__ void ldb_frag_nk(uint32_t (&b)[4], const __nv_bfloat16* s, int n0, int kk, int lane) {
  const int r = n0 + ((lane >> 4) << 3) + (lane & 7);
  const int c = kk * 2 + ((lane >> 3) & 1);
  ldsm_x4(b, s + swz(r, c));
}
// B fragments for two n8 tiles from a [k x n] row-major tile (k rows k0..k0+15, n cols n0..n0+15).
__device__ __forceinline__ void ldb_frag_kn(uint32_t (&b)[4], const __nv_bfloat16* s, int k0, int n0, int lane) {
  const int r = k0 + (((lane >> 3) & 1) << 3) + (lane & 7);
  const int c = (n0 >> 3) + (lane >> 4);
  ldsm_x4_t(b, s + swz(r, c));
}

}  // namespace

// ------------------------------------------------------------------ forward
__global__ void __launch_bounds__(kWarps * 32)
    attn_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out, float* __restrict__ lse,
                    int S, int heads, float scale_log2) {
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int H = heads * kD;
  const long long ld = 3LL * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row_base = b * S;  // first token row of this sequence
  const int q0 = qt * kTileQ;

  __shared__ __align__(128) __nv_bfloat16 sQ[64 * 64];
  __shared__ __align__(128) __nv_bfloat16 sK[2][64 * 64];
  __shared__ __align__(128) __nv_bfloat16 sV[2][64 * 64];

  const __nv_bfloat16* gq = qkv + static_cast<long long>(row_base) * ld + h * kD;
  const __nv_bfloat16* gk = gq + H;
  const __nv_bfloat16* gv = gq + 2 * H;

  load_tile(sQ, gq, ld, q0, S, 0, tid, kWarps * 32);
  load_tile(sK[0], gk, ld, 0, S, 0, tid, kWarps * 32);
  load_tile(sV[0], gv, ld, 0, S, 0, tid, kWarps * 32);
  cp_async_commit();

  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qa[4][4];

  const int nkt = (S + kTileK - 1) / kTileK;
  for (int kt = 0; kt < nkt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < nkt) {
      load_tile(sK[buf ^ 1], gk, ld, (kt + 1) * kTileK, S, 0, tid, kWarps * 32);
      load_tile(sV[buf ^ 1], gv, ld, (kt + 1) * kTileK, S, 0, tid, kWarps * 32);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) lda_frag(qa[kk], sQ, warp * 16, kk, lane);
    }
    // S = Q K^T  (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t bb[4];
        ldb_frag_nk(bb, sK[buf], jj * 16, kk, lane);
        mma16816(s[2 * jj], qa[kk], bb[0], bb[1]);
        mma16816(s[2 * jj + 1], qa[kk], bb[2], bb[3]);
      }
    }
    // mask keys past the end of the sequence
    const int kbase = kt * kTileK;
    if (kbase + kTileK > S) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int kc = kbase + j * 8 + 2 * (lane & 3);
        if (kc >= S) { s[j][0] = -INFINITY; s[j][2] = -INFINITY; }
        if (kc + 1 >= S) { s[j][1] = -INFINITY; s[j][3] = -INFINITY; }
      }
    }
    // online softmax (rows g and g+8 of this warp's 16)
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]) * scale_log2);
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]) * scale_log2);
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float a0 = exp2f(m0 - mx0), a1 = exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pa[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = exp2f(s[j][0] * scale_log2 - mx0), p1 = exp2f(s[j][1] * scale_log2 - mx0);
      const float p2 = exp2f(s[j][2] * scale_log2 - mx1), p3 = exp2f(s[j][3] * scale_log2 - mx1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      const int kk = j >> 1;
      if ((j & 1) == 0) {
        pa[kk][0] = pack_bf16x2(p0, p1);
        pa[kk][1] = pack_bf16x2(p2, p3);
      } else {
        pa[kk][2] = pack_bf16x2(p0, p1);
        pa[kk][3] = pack_bf16x2(p2, p3);
      }
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= a0; o[j][1] *= a0;
      o[j][2] *= a1; o[j][3] *= a1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t bb[4];
        ldb_frag_kn(bb, sV[buf], kk * 16, jj * 16, lane);
        mma16816(o[2 * jj], pa[kk], bb[0], bb[1]);
        mma16816(o[2 * jj + 1], pa[kk], bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const int r0 = q0 + warp * 16 + (lane >> 2);
  const int r1 = r0 + 8;
  __nv_bfloat16* go = out + static_cast<long long>(row_base) * H + h * kD;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = j * 8 + 2 * (lane & 3);
    if (r0 < S)
      *reinterpret_cast<uint32_t*>(go + static_cast<long long>(r0) * H + c) = pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
    if (r1 < S)
      *reinterpret_cast<uint32_t*>(go + static_cast<long long>(r1) * H + c) = pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
  }
  if ((lane & 3) == 0) {
    const float ln2 = 0.69314718055994531f;
    float* gl = lse + (static_cast<long long>(b) * heads + h) * S;
    if (r0 < S) gl[r0] = (m0 + log2f(l0)) * ln2;
    if (r1 < S) gl[r1] = (m1 + log2f(l1)) * ln2;
  }
}

// ------------------------------------------------------------------ backward
// Backward pre-pass: D[b, h, s] = sum_d dO[s, h*64 + d] * O[s, h*64 + d], and the fp32 dQ
// accumulator slice of (s, h) is zeroed (when given).  Eight threads per (row, head), 16
// bytes of dO and O each, so a warp reads four consecutive 128-byte head slices.
__global__ void attn_bwd_dot_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                    float* __restrict__ D, float* __restrict__ dq_acc, int M, int S, int heads) {
  const int H = heads * kD;
  const long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long pair = t >> 3;
  const int sub = static_cast<int>(t & 7);
  if (pair >= static_cast<long long>(M) * heads) return;  // whole groups of eight leave together
  const int row = static_cast<int>(pair / heads), h = static_cast<int>(pair % heads);
  const long long off = static_cast<long long>(row) * H + h * kD + sub * 8;
  const uint4 a = *reinterpret_cast<const uint4*>(dout + off);
  const uint4 c = *reinterpret_cast<const uint4*>(out + off);
  const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, cw[4] = {c.x, c.y, c.z, c.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = unpack_bf16x2(aw[i]), y = unpack_bf16x2(cw[i]);
    s = fmaf(x.x, y.x, s);
    s = fmaf(x.y, y.y, s);
  }
  const unsigned mask = 0xffu << (threadIdx.x & 24);
  s += __shfl_xor_sync(mask, s, 1);
  s += __shfl_xor_sync(mask, s, 2);
  s += __shfl_xor_sync(mask, s, 4);
  if (sub == 0) {
    const int b = row / S, sidx = row % S;
    D[(static_cast<long long>(b) * heads + h) * S + sidx] = s;
  }
  if (dq_acc != nullptr) {
    float4* z = reinterpret_cast<float4*>(dq_acc + off);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// One CTA per (key tile of 64, head, batch); 4 warps x 16 keys.  Loops over query tiles.
// dK, dV accumulate in registers; dQ (scaled) accumulates in an fp32 buffer with atomics.
__global__ void __launch_bounds__(kWarps * 32)
    attn_bwd_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ dout,
                    const float* __restrict__ lse, const float* __restrict__ Dd, float* __restrict__ dq_acc,
                    __nv_bfloat16* __restrict__ dqkv, int S, int heads, float scale, float scale_log2) {
  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int H = heads * kD;
  const long long ld = 3LL * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row_base = b * S;
  const int k0 = kt * kTileK;

  extern __shared__ __align__(128) uint8_t attn_bwd_smem[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(attn_bwd_smem);
  __nv_bfloat16* sV = sK + 64 * 64;
  __nv_bfloat16 (*sQ)[64 * 64] = reinterpret_cast<__nv_bfloat16 (*)[64 * 64]>(sV + 64 * 64);
  __nv_bfloat16 (*sdO)[64 * 64] = reinterpret_cast<__nv_bfloat16 (*)[64 * 64]>(sV + 3 * 64 * 64);
  __nv_bfloat16* sdS = sV + 5 * 64 * 64;  // dS^T [keys x queries]
  float (*sL)[64] = reinterpret_cast<float (*)[64]>(sdS + 64 * 64);
  float (*sD)[64] = sL + 2;

  const __nv_bfloat16* gq = qkv + static_cast<long long>(row_base) * ld + h * kD;
  const __nv_bfloat16* gk = gq + H;
  const __nv_bfloat16* gv = gq + 2 * H;
  const __nv_bfloat16* gdo = dout + static_cast<long long>(row_base) * H + h * kD;
  const float* gl = lse + (static_cast<long long>(b) * heads + h) * S;
  const float* gD = Dd + (static_cast<long long>(b) * heads + h) * S;

  load_tile(sK, gk, ld, k0, S, 0, tid, kWarps * 32);
  load_tile(sV, gv, ld, k0, S, 0, tid, kWarps * 32);
  load_tile(sQ[0], gq, ld, 0, S, 0, tid, kWarps * 32);
  load_tile(sdO[0], gdo, H, 0, S, 0, tid, kWarps * 32);
  cp_async_commit();
  if (tid < 64) {
    sL[0][tid] = tid < S ? gl[tid] : 0.f;
    sD[0][tid] = tid < S ? gD[tid] : 0.f;
  }

  float dk[8][4], dv[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    dk[j][0] = dk[j][1] = dk[j][2] = dk[j][3] = 0.f;
    dv[j][0] = dv[j][1] = dv[j][2] = dv[j][3] = 0.f;
  }
  uint32_t ka[4][4], va[4][4];
  const int key_r0 = k0 + warp * 16 + (lane >> 2);  // this thread's key rows (r0, r0+8)
  const bool key0_ok = key_r0 < S, key1_ok = key_r0 + 8 < S;

  const int nqt = (S + kTileQ - 1) / kTileQ;
  for (int qt = 0; qt < nqt; ++qt) {
    const int buf = qt & 1;
    if (qt + 1 < nqt) {
      load_tile(sQ[buf ^ 1], gq, ld, (qt + 1) * kTileQ, S, 0, tid, kWarps * 32);
      load_tile(sdO[buf ^ 1], gdo, H, (qt + 1) * kTileQ, S, 0, tid, kWarps * 32);
      cp_async_commit();
      if (tid < 64) {
        const int qi = (qt + 1) * kTileQ + tid;
        sL[buf ^ 1][tid] = qi < S ? gl[qi] : 0.f;
        sD[buf ^ 1][tid] = qi < S ? gD[qi] : 0.f;
      }
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (qt == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        lda_frag(ka[kk], sK, warp * 16, kk, lane);
        lda_frag(va[kk], sV, warp * 16, kk, lane);
      }
    }
    const int q0 = qt * kTileQ;
    // S^T = K Q^T and dP^T = V dO^T  (16 keys x 64 queries per warp)
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      st[j][0] = st[j][1] = st[j][2] = st[j][3] = 0.f;
      dpt[j][0] = dpt[j][1] = dpt[j][2] = dpt[j][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t bq[4], bo[4];
        ldb_frag_nk(bq, sQ[buf], jj * 16, kk, lane);
        ldb_frag_nk(bo, sdO[buf], jj * 16, kk, lane);
        mma16816(st[2 * jj], ka[kk], bq[0], bq[1]);
        mma16816(st[2 * jj + 1], ka[kk], bq[2], bq[3]);
        mma16816(dpt[2 * jj], va[kk], bo[0], bo[1]);
        mma16816(dpt[2 * jj + 1], va[kk], bo[2], bo[3]);
      }
    }
    // P^T = exp(S^T * scale - lse_q); dS^T = P^T * (dP^T - D_q)
    uint32_t pa[4][4], dsa[4][4];
    const float ln2inv = 1.4426950408889634f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int qc = j * 8 + 2 * (lane & 3);
      const bool q0ok = q0 + qc < S, q1ok = q0 + qc + 1 < S;
      const float L0 = sL[buf][qc] * ln2inv, L1 = sL[buf][qc + 1] * ln2inv;
      const float D0 = sD[buf][qc], D1 = sD[buf][qc + 1];
      float p[4];
      p[0] = (key0_ok && q0ok) ? exp2f(st[j][0] * scale_log2 - L0) : 0.f;
      p[1] = (key0_ok && q1ok) ? exp2f(st[j][1] * scale_log2 - L1) : 0.f;
      p[2] = (key1_ok && q0ok) ? exp2f(st[j][2] * scale_log2 - L0) : 0.f;
      p[3] = (key1_ok && q1ok) ? exp2f(st[j][3] * scale_log2 - L1) : 0.f;
      // P rounded to bf16 feeds dV; dS uses the same rounded P.
      const uint32_t p01 = pack_bf16x2(p[0], p[1]), p23 = pack_bf16x2(p[2], p[3]);
      const float2 pr01 = unpack_bf16x2(p01), pr23 = unpack_bf16x2(p23);
      const float ds0 = pr01.x * (dpt[j][0] - D0), ds1 = pr01.y * (dpt[j][1] - D1);
      const float ds2 = pr23.x * (dpt[j][2] - D0), ds3 = pr23.y * (dpt[j][3] - D1);
      const uint32_t d01 = pack_bf16x2(ds0, ds1), d23 = pack_bf16x2(ds2, ds3);
      const int kk = j >> 1;
      if ((j & 1) == 0) {
        pa[kk][0] = p01; pa[kk][1] = p23;
        dsa[kk][0] = d01; dsa[kk][1] = d23;
      } else {
        pa[kk][2] = p01; pa[kk][3] = p23;
        dsa[kk][2] = d01; dsa[kk][3] = d23;
      }
      // stash dS^T for the dQ product: rows = keys (warp*16 + g, +8), cols = queries
      const int kr = warp * 16 + (lane >> 2);
      *reinterpret_cast<uint32_t*>(sdS + swz(kr, qc >> 3) + (qc & 7)) = d01;
      *reinterpret_cast<uint32_t*>(sdS + swz(kr + 8, qc >> 3) + (qc & 7)) = d23;
    }
    // dV += P^T dO ; dK += dS^T Q    (16 keys x 64 d per warp, k = queries)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t bo[4], bq[4];
        ldb_frag_kn(bo, sdO[buf], kk * 16, jj * 16, lane);
        ldb_frag_kn(bq, sQ[buf], kk * 16, jj * 16, lane);
        mma16816(dv[2 * jj], pa[kk], bo[0], bo[1]);
        mma16816(dv[2 * jj + 1], pa[kk], bo[2], bo[3]);
        mma16816(dk[2 * jj], dsa[kk], bq[0], bq[1]);
        mma16816(dk[2 * jj + 1], dsa[kk], bq[2], bq[3]);
      }
    }
    __syncthreads();  // sdS complete
    // dQ[q, d] += sum_keys dS[q, key] K[key, d]  (warp: 16 queries x 64 d, k = keys)
    {
      float dqv[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) dqv[j][0] = dqv[j][1] = dqv[j][2] = dqv[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        // A = dS [q x keys]: from dS^T stored [keys x q] via transposed ldmatrix
        uint32_t a[4];
        {
          const int key = kk * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int qch = ((warp * 16) >> 3) + ((lane >> 3) & 1);
          ldsm_x4_t(a, sdS + swz(key, qch));
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          uint32_t bk[4];
          ldb_frag_kn(bk, sK, kk * 16, jj * 16, lane);
          mma16816(dqv[2 * jj], a, bk[0], bk[1]);
          mma16816(dqv[2 * jj + 1], a, bk[2], bk[3]);
        }
      }
      const int qr0 = q0 + warp * 16 + (lane >> 2);
      float* gdq = dq_acc + static_cast<long long>(row_base) * H + h * kD;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = j * 8 + 2 * (lane & 3);
        if (qr0 < S)
          atomicAdd(reinterpret_cast<float2*>(gdq + static_cast<long long>(qr0) * H + c),
                    make_float2(dqv[j][0] * scale, dqv[j][1] * scale));
        if (qr0 + 8 < S)
          atomicAdd(reinterpret_cast<float2*>(gdq + static_cast<long long>(qr0 + 8) * H + c),
                    make_float2(dqv[j][2] * scale, dqv[j][3] * scale));
      }
    }
    __syncthreads();  // buffers reused by the next prefetch
  }
  // write dK (scaled) and dV
  __nv_bfloat16* gdk = dqkv + static_cast<long long>(row_base) * ld + H + h * kD;
  __nv_bfloat16* gdv = gdk + H;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = j * 8 + 2 * (lane & 3);
    if (key0_ok) {
      *reinterpret_cast<uint32_t*>(gdk + static_cast<long long>(key_r0) * ld + c) = pack_bf16x2(dk[j][0] * scale, dk[j][1] * scale);
      *reinterpret_cast<uint32_t*>(gdv + static_cast<long long>(key_r0) * ld + c) = pack_bf16x2(dv[j][0], dv[j][1]);
    }
    if (key1_ok) {
      *reinterpret_cast<uint32_t*>(gdk + static_cast<long long>(key_r0 + 8) * ld + c) = pack_bf16x2(dk[j][2] * scale, dk[j][3] * scale);
      *reinterpret_cast<uint32_t*>(gdv + static_cast<long long>(key_r0 + 8) * ld + c) = pack_bf16x2(dv[j][2], dv[j][3]);
    }
  }
}

// dqkv[:, 0:H] = bf16(dq_acc)
__global__ void attn_dq_convert_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv, long long M,
                                       int H) {
  const long long i4 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long n4 = M * H / 4;
  if (i4 >= n4) return;
  const long long e = i4 * 4;
  const long long row = e / H;
  const int col = static_cast<int>(e % H);
  const float4 v = reinterpret_cast<const float4*>(dq_acc)[i4];
  *reinterpret_cast<uint2*>(dqkv + row * 3LL * H + col) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

// ------------------------------------------------------------------ host side
void attn_bwd_dot_launch(const torch::Tensor& dout, const torch::Tensor& out, torch::Tensor D, torch::Tensor dq_acc,
                         int64_t M, int64_t S, int64_t heads) {
  const long long threads_total = M * heads * 8;
  const int threads = 256;
  const long long blocks = (threads_total + threads - 1) / threads;
  attn_bwd_dot_kernel<<<static_cast<unsigned>(blocks), threads, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
      D.data_ptr<float>(), dq_acc.defined() ? dq_acc.data_ptr<float>() : nullptr, static_cast<int>(M),
      static_cast<int>(S), static_cast<int>(heads));
  REVPP_CHECK_LAUNCH();
}

void attn_dq_convert_launch(const torch::Tensor& dq_acc, torch::Tensor dqkv, int64_t M, int64_t H) {
  const long long n4 = M * H / 4;
  const int threads = 256;
  attn_dq_convert_kernel<<<static_cast<unsigned>((n4 + threads - 1) / threads), threads, 0, cur_stream()>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), M, static_cast<int>(H));
  REVPP_CHECK_LAUNCH();
}

void attn_fwd(const torch::Tensor& qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t S, int64_t heads) {
  check_cuda_bf16(qkv, "qkv");
  check_cuda_bf16(out, "out");
  check_cuda_f32(lse, "lse");
  const int64_t H = heads * kD;
  REVPP_CHECK(qkv.is_contiguous() && qkv.size(0) == B * S && qkv.size(1) == 3 * H, "qkv must be [B*S, 3H]");
  REVPP_CHECK(out.is_contiguous() && out.size(0) == B * S && out.size(1) == H, "out must be [B*S, H]");
  REVPP_CHECK(lse.numel() >= B * heads * S, "lse too small");
  c10::cuda::CUDAGuard guard(qkv.device());
  const float scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(kD)));
  dim3 grid(static_cast<unsigned>((S + kTileQ - 1) / kTileQ), static_cast<unsigned>(heads), static_cast<unsigned>(B));
  attn_fwd_kernel<<<grid, kWarps * 32, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      lse.data_ptr<float>(), static_cast<int>(S), static_cast<int>(heads), scale_log2);
  REVPP_CHECK_LAUNCH();
}

// dq_acc (fp32 [B*S, H]) and D (fp32 [B, heads, S]) are scratch buffers supplied by the caller.
void attn_bwd(const torch::Tensor& qkv, const torch::Tensor& out, const torch::Tensor& dout, const torch::Tensor& lse,
              torch::Tensor dqkv, torch::Tensor dq_acc, torch::Tensor Dbuf, int64_t B, int64_t S, int64_t heads) {
  check_cuda_bf16(qkv, "qkv");
  check_cuda_bf16(out, "out");
  check_cuda_bf16(dout, "dout");
  check_cuda_bf16(dqkv, "dqkv");
  check_cuda_f32(lse, "lse");
  check_cuda_f32(dq_acc, "dq_acc");
  check_cuda_f32(Dbuf, "D");
  const int64_t H = heads * kD;
  const int64_t M = B * S;
  REVPP_CHECK(qkv.is_contiguous() && qkv.size(0) == M && qkv.size(1) == 3 * H, "qkv must be [B*S, 3H]");
  REVPP_CHECK(dqkv.is_contiguous() && dqkv.size(0) == M && dqkv.size(1) == 3 * H, "dqkv must be [B*S, 3H]");
  REVPP_CHECK(out.is_contiguous() && dout.is_contiguous() && out.numel() == M * H && dout.numel() == M * H,
              "out/dout must be [B*S, H]");
  REVPP_CHECK(dq_acc.numel() >= M * H && Dbuf.numel() >= B * heads * S, "scratch too small");
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t st = cur_stream();
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(kD)));
  const float scale_log2 = static_cast<float>(1.4426950408889634) * scale;
  attn_bwd_dot_launch(dout, out, Dbuf, dq_acc, M, S, heads);  // D, and dq_acc = 0
  dim3 grid(static_cast<unsigned>((S + kTileK - 1) / kTileK), static_cast<unsigned>(heads), static_cast<unsigned>(B));
  constexpr int smem = 7 * 64 * 64 * 2 + 4 * 64 * 4;
  static int configured_for = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_for != dev) {
    REVPP_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured_for = dev;
  }
  attn_bwd_kernel<<<grid, kWarps * 32, smem, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      lse.data_ptr<float>(), Dbuf.data_ptr<float>(), dq_acc.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), static_cast<int>(S), static_cast<int>(heads), scale, scale_log2);
  REVPP_CHECK_LAUNCH();
  {
    const long long n4 = M * H / 4;
    const int threads = 256;
    attn_dq_convert_kernel<<<static_cast<unsigned>((n4 + threads - 1) / threads), threads, 0, st>>>(
        dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), M, static_cast<int>(H));
    REVPP_CHECK_LAUNCH();
  }
}

}  // namespace revpp
