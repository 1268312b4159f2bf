// Flash attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
// Head dim 64; same interface and numerics as attn_fwd in attention.cu (qkv packed as
// nn.MultiheadAttention's in_proj output, o [B*S, H] bf16, lse [B, heads, S] fp32).
//
// One CTA per (query tile of 128 rows, head, sequence); 64-key tiles.
//   warp 0     : TMA producer - Q once, then K_j / V_j into a 3-deep ring (no multicast)
//   warp 1     : TMEM allocator and MMA issuer (one thread):
//                  S_j  = Q K_j^T   (M 128, N 64, K 64)  -> TMEM S[j % 2]
//                  PV_j = P_j V_j   (M 128, N 64, K 64)  -> TMEM PV[j % 2]
//                S_{j+1} is issued before waiting for P_j, so the tensor core works on the
//                next scores while the softmax warps handle the current ones.
//   warps 2-5  : softmax, one thread per query row: S row from TMEM, online max / sum in
//                fp32 (exp2 with the 1/sqrt(d) * log2(e) scale folded in), P_j as bf16 into a
//                128-byte-swizzled smem tile (the MMA's A operand), and O accumulated in
//                registers: O = O * alpha_{j-1} + PV_{j-1}.
// Shared memory ~97 KB and 256 TMEM columns, so two CTAs share an SM.
#include "common.cuh"
#include "host.h"

namespace revpp {

namespace {
constexpr int kQ = 128;      // query rows per CTA
constexpr int kKV = 64;      // keys per tile
constexpr int kDh = 64;      // head dim
constexpr int kStages = 3;   // K/V ring depth
constexpr int kThreads = 192;
constexpr uint32_t kQBytes = kQ * kDh * 2;     // 16 KB
constexpr uint32_t kKVBytes = kKV * kDh * 2;   // 8 KB (one of K or V)
constexpr uint32_t kPBytes = kQ * kKV * 2;     // 16 KB
constexpr uint32_t kTmemCols = 256;            // S[2] (64 each) + PV[2] (64 each)
constexpr uint32_t kIdescS = idesc_bf16(kQ, kKV, false, false);
constexpr uint32_t kIdescPV = idesc_bf16(kQ, kDh, false, true);

struct SmemLayout {
  // offsets from the 1024-aligned base
  static constexpr uint32_t q = 0;
  static constexpr uint32_t k = q + kQBytes;                      // kStages x 8 KB
  static constexpr uint32_t v = k + kStages * kKVBytes;           // kStages x 8 KB
  static constexpr uint32_t p = v + kStages * kKVBytes;           // 2 x 16 KB
  static constexpr uint32_t bars = p + 2 * kPBytes;
  static constexpr uint32_t total = bars + 256;
};
}  // namespace

struct AttnTcArgs {
  __nv_bfloat16* out;
  float* lse;
  int S, heads;
  float scale_log2;
  int* status;
};

__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                       const AttnTcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SmemLayout::bars);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + 1;              // [kStages]
  uint64_t* kv_empty = kv_full + kStages;   // [kStages]
  uint64_t* s_full = kv_empty + kStages;    // [2]
  uint64_t* s_empty = s_full + 2;           // [2]
  uint64_t* p_full = s_empty + 2;           // [2]
  uint64_t* p_empty = p_full + 2;           // [2]
  uint64_t* pv_full = p_empty + 2;          // [2]
  uint64_t* pv_empty = pv_full + 2;         // [2]
  uint64_t* drain = pv_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int S = args.S;
  const int H = args.heads * kDh;
  const int row0 = b * S;                 // first token row of this sequence
  const int q0 = qt * kQ;
  const int nkv = (S + kKV - 1) / kKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
      mbar_init(&pv_full[i], 1);
      mbar_init(&pv_empty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      mbar_arrive_expect_tx(q_full, kQBytes);
      tma_load_2d(smem + SmemLayout::q, &tmQ, q_full, h * kDh, row0 + q0);
      uint32_t issued = 0, issued_par = 0;
      for (int j = 0; j < nkv; ++j) {
        const int st = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, args.status, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kKVBytes);
        tma_load_2d(smem + SmemLayout::k + st * kKVBytes, &tmKV, &kv_full[st], H + h * kDh, row0 + j * kKV);
        tma_load_2d(smem + SmemLayout::v + st * kKVBytes, &tmKV, &kv_full[st], 2 * H + h * kDh, row0 + j * kKV);
        issued |= 1u << st;
        issued_par = (issued_par & ~(1u << st)) | (ph << st);
      }
      if (*abort_flag) {
        // let in-flight copies land before the CTA exits
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
        for (int s = 0; s < kStages; ++s) {
          if (!(issued & (1u << s))) continue;
          const uint64_t t1 = globaltimer_ns();
          while (!mbar_try_wait(&kv_full[s], (issued_par >> s) & 1u) && globaltimer_ns() - t1 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t q_addr = smem_u32(smem + SmemLayout::q);
      const uint32_t k_addr = smem_u32(smem + SmemLayout::k);
      const uint32_t v_addr = smem_u32(smem + SmemLayout::v);
      const uint32_t p_addr = smem_u32(smem + SmemLayout::p);
      bool ok = mbar_wait(q_full, 0, args.status, abort_flag);
      auto issue_pv = [&](int j) -> bool {
        const int pb = j & 1;
        const uint32_t par = (j >> 1) & 1;
        if (!mbar_wait(&p_full[pb], par, args.status, abort_flag)) return false;
        if (!mbar_wait(&pv_empty[pb], par ^ 1u, args.status, abort_flag)) return false;
        tc_fence_after();
        const int st = j % kStages;
        const uint32_t d = tmem + 128 + pb * kDh;
#pragma unroll
        for (int k = 0; k < kKV / 16; ++k) {
          const uint64_t ad = sdesc_sw128(p_addr + pb * kPBytes + k * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(v_addr + st * kKVBytes + k * 2048, 8192, 1024);
          umma_bf16_ss(d, ad, bd, kIdescPV, k > 0 ? 1u : 0u);
        }
        umma_commit(&pv_full[pb]);
        umma_commit(&p_empty[pb]);
        umma_commit(&kv_empty[st]);
        return true;
      };
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        const int sb = j & 1;
        if (!mbar_wait(&kv_full[st], ph, args.status, abort_flag)) break;
        if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1u, args.status, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + sb * kKV;
#pragma unroll
        for (int k = 0; k < kDh / 16; ++k) {
          const uint64_t ad = sdesc_sw128(q_addr + k * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_addr + st * kKVBytes + k * 32, 16, 1024);
          umma_bf16_ss(d, ad, bd, kIdescS, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && nkv >= 1) issue_pv(nkv - 1);
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kIntraKernelTimeoutNs) {
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;           // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* p_base = smem + SmemLayout::p;
    float o[kDh];
#pragma unroll
    for (int i = 0; i < kDh; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    const float sl2 = args.scale_log2;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int sb = j & 1;
      const uint32_t par = (j >> 1) & 1;
      if (!mbar_wait(&s_full[sb], par, args.status, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld32(tmem + lane_off + sb * kKV, sr[0]);
      tmem_ld32(tmem + lane_off + sb * kKV + 32, sr[1]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);
      float sv[kKV];
#pragma unroll
      for (int c = 0; c < kKV; ++c) sv[c] = __uint_as_float(sr[c >> 5][c & 31]) * sl2;
      const int kbase = j * kKV;
      if (kbase + kKV > S) {
#pragma unroll
        for (int c = 0; c < kKV; ++c)
          if (kbase + c >= S) sv[c] = -INFINITY;
      }
      float mx = m;
#pragma unroll
      for (int c = 0; c < kKV; ++c) mx = fmaxf(mx, sv[c]);
      const float alpha = exp2f(m - mx);
      float rs = 0.f;
      l *= alpha;
      m = mx;
      // P_j -> smem (A operand of P V, 128-byte swizzle: 16-byte chunk c of row r at c ^ (r & 7))
      if (!mbar_wait(&p_empty[sb], par ^ 1u, args.status, abort_flag)) {
        ok = false;
        break;
      }
      uint8_t* prow = p_base + sb * kPBytes + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = exp2f(sv[8 * c + 2 * e] - mx), p1 = exp2f(sv[8 * c + 2 * e + 1] - mx);
          rs += p0 + p1;
          w[e] = pack_bf16x2(p0, p1);
        }
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l += rs;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
      // fold in PV_{j-1}
      if (j >= 1) {
        const int pb = (j - 1) & 1;
        if (!mbar_wait(&pv_full[pb], ((j - 1) >> 1) & 1, args.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t pv[2][32];
        tmem_ld32(tmem + lane_off + 128 + pb * kDh, pv[0]);
        tmem_ld32(tmem + lane_off + 128 + pb * kDh + 32, pv[1]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pv_empty[pb]);
#pragma unroll
        for (int i = 0; i < kDh; ++i) o[i] = o[i] * alpha_prev + __uint_as_float(pv[i >> 5][i & 31]);
      }
      alpha_prev = alpha;
    }
    if (ok && nkv >= 1) {
      const int pb = (nkv - 1) & 1;
      if (mbar_wait(&pv_full[pb], ((nkv - 1) >> 1) & 1, args.status, abort_flag)) {
        tc_fence_after();
        uint32_t pv[2][32];
        tmem_ld32(tmem + lane_off + 128 + pb * kDh, pv[0]);
        tmem_ld32(tmem + lane_off + 128 + pb * kDh + 32, pv[1]);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < kDh; ++i) o[i] = o[i] * alpha_prev + __uint_as_float(pv[i >> 5][i & 31]);
        const int q = q0 + r;
        if (q < S) {
          const float inv = 1.f / l;
          uint4* dst = reinterpret_cast<uint4*>(args.out + (static_cast<long long>(row0) + q) * H + h * kDh);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            dst[c] = make_uint4(pack_bf16x2(o[8 * c] * inv, o[8 * c + 1] * inv),
                                pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                                pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                                pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
          }
          args.lse[(static_cast<long long>(b) * args.heads + h) * S + q] = (m + log2f(l)) * 0.69314718055994531f;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

void attn_fwd_tc(const torch::Tensor& qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t S,
                 int64_t heads) {
  check_cuda_bf16(qkv, "qkv");
  check_cuda_bf16(out, "out");
  check_cuda_f32(lse, "lse");
  const int64_t H = heads * kDh;
  REVPP_CHECK(qkv.is_contiguous() && qkv.size(0) == B * S && qkv.size(1) == 3 * H, "qkv must be [B*S, 3H]");
  REVPP_CHECK(out.is_contiguous() && out.size(0) == B * S && out.size(1) == H, "out must be [B*S, H]");
  REVPP_CHECK(lse.numel() >= B * heads * S, "lse too small");
  c10::cuda::CUDAGuard guard(qkv.device());
  const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  const CUtensorMap tq = make_tmap_2d(qkv.data_ptr(), bf, 2, 3 * H, B * S, 3 * H * 2, 64, kQ, sw);
  const CUtensorMap tkv = make_tmap_2d(qkv.data_ptr(), bf, 2, 3 * H, B * S, 3 * H * 2, 64, kKV, sw);
  AttnTcArgs a;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.S = static_cast<int>(S);
  a.heads = static_cast<int>(heads);
  a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(kDh)));
  a.status = status_device_ptr();
  constexpr int smem = SmemLayout::total + 1024;
  static int configured_for = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_for != dev) {
    REVPP_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured_for = dev;
  }
  dim3 grid(static_cast<unsigned>((S + kQ - 1) / kQ), static_cast<unsigned>(heads), static_cast<unsigned>(B));
  attn_fwd_tc_kernel<<<grid, kThreads, smem, cur_stream()>>>(tq, tkv, a);
  REVPP_CHECK_LAUNCH();
}

}  // namespace revpp
