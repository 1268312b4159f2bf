// Persistent flash attention forward on the 5th-generation tensor cores (tcgen05 + TMEM +
// TMA), head dim 64; interface and numerics of attn_fwd_tc (attention_tc.cu): qkv packed as
// nn.MultiheadAttention's in_proj output [B*S, 3H], o [B*S, H] bf16, lse [B, heads, S] fp32.
//
// With head dim 64 each score costs 256 tensor-core FLOPs (Q K^T and P V) but one exp2 on the
// MUFU, whose rate is half the tensor core's per score: the kernel is bounded by how
// busily the softmax warps keep the MUFU fed.  The non-persistent kernel (two groups
// splitting the key tiles of one query tile, a single S and P buffer per group) left the
// softmax warps waiting on their next scores or on the tensor core freeing their P tile,
// and paid a per-CTA prologue and merge.  Here:
//   * one CTA per SM walks work items (2 query tiles of 128 rows of one head and sequence;
//     items of a sequence are consecutive, so K / V stay in L2);
//   * softmax group w (4 warps, one query row per thread) owns query tile w of the item and
//     runs over all its key tiles: no merge, each group normalises and stores its rows;
//   * TMEM (all 512 columns): S[w][2] double-buffered scores and O[w][2] double-buffered
//     outputs, so a group's next scores are computed while it works on the current ones,
//     and the next item's P V runs while the group stores the previous item's output;
//   * P[w][2] double-buffered in shared memory: writing P_t waits for P V of tile t-2 only;
//   * Q of the next item is loaded while the current item runs (Q[2 items][2 groups]).
// The reference maximum of a row is raised only when a tile maximum exceeds it by more
// than 8 (log2 units), with O rescaled through tcgen05.ld / st after the group's previous
// P V has landed (as in attn_fwd_tc).
//   warp 0    : TMA producer (one thread): Q, then K_u / V_u of the flat tile sequence of
//               this CTA's items into a 4-deep ring (no multicast)
//   warp 1    : TMEM allocator and MMA issuer (one thread): S two tiles ahead of P V, per group
//   warps 2-5 : softmax group 0; warps 6-9: softmax group 1
// Every wait is bounded; on a timeout the kernel records the status bit and unwinds.
#include "common.cuh"
#include "host.h"

namespace revpp {
namespace {
namespace fa {
constexpr int kQ = 128;
constexpr int kKV = 64;
constexpr int kDh = 64;
constexpr int kStages = 4;
constexpr int kThreads = 320;
constexpr uint32_t kQBytes = kQ * kDh * 2;    // 16 KB
constexpr uint32_t kKVBytes = kKV * kDh * 2;  // 8 KB
constexpr uint32_t kPBytes = kQ * kKV * 2;    // 16 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 256;  // S[w][b] at 128 w + 64 b, O[w][b] at 256 + 128 w + 64 b
constexpr float kRescaleThreshold = 8.0f;
constexpr uint32_t kIdescS = idesc_bf16(kQ, kKV, false, false);
constexpr uint32_t kIdescPV = idesc_bf16(kQ, kDh, false, true);

struct Smem {
  static constexpr uint32_t q = 0;                          // [item buffer][group] x 16 KB
  static constexpr uint32_t k = q + 4 * kQBytes;            // kStages x 8 KB
  static constexpr uint32_t v = k + kStages * kKVBytes;     // kStages x 8 KB
  static constexpr uint32_t p = v + kStages * kKVBytes;     // [group][buffer] x 16 KB
  static constexpr uint32_t bars = p + 4 * kPBytes;
  static constexpr uint32_t total = bars + 512;
};

struct Args {
  __nv_bfloat16* out;
  float* lse;
  int S, heads, npairs, num_items, nkv;
  float scale_log2;
  int* status;
};

struct Item {
  int b, h, q0;     // sequence, head, first query row of group 0's tile
  bool valid1;      // group 1's tile starts inside the sequence
};
__device__ __forceinline__ Item item_of(const Args& a, int it) {
  Item r;
  const int p = it % a.npairs;
  const int hb = it / a.npairs;
  r.h = hb % a.heads;
  r.b = hb / a.heads;
  r.q0 = 2 * p * kQ;
  r.valid1 = r.q0 + kQ < a.S;
  return r;
}
}  // namespace fa
}  // namespace

__global__ void __launch_bounds__(fa::kThreads, 1)
    attn_fwd_persistent_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                               const fa::Args args) {
  using namespace fa;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Smem::bars);
  uint64_t* q_full = bar;                  // [2] item buffers
  uint64_t* q_empty = q_full + 2;          // [2]
  uint64_t* k_full = q_empty + 2;          // [kStages]
  uint64_t* k_empty = k_full + kStages;    // [kStages]
  uint64_t* v_full = k_empty + kStages;    // [kStages]
  uint64_t* v_empty = v_full + kStages;    // [kStages]
  uint64_t* s_full = v_empty + kStages;    // [group][2]
  uint64_t* s_empty = s_full + 4;          // [group][2]
  uint64_t* p_full = s_empty + 4;          // [group][2]
  uint64_t* p_empty = p_full + 4;          // [group][2]  (P V of that buffer done)
  uint64_t* o_full = p_empty + 4;          // [group][2]
  uint64_t* o_empty = o_full + 4;          // [group][2]
  uint64_t* drain = o_empty + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = args.S;
  const int H = args.heads * kDh;
  const int nkv = args.nkv;
  // this CTA's items: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_items = args.num_items > static_cast<int>(blockIdx.x)
                           ? (args.num_items - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                           : 0;
  const int total_u = my_items * nkv;  // flat key-tile sequence of this CTA
  auto item_at = [&](int il) { return item_of(args, static_cast<int>(blockIdx.x) + il * static_cast<int>(gridDim.x)); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
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
    if (lane == 0 && my_items > 0) {
      // ---------------------------------------------------------------- producer
      uint32_t pending = 0, pending_par = 0;  // bits: K stages, V stages, Q buffers (abort drain)
      auto load_q = [&](int il) -> bool {
        const int qb = il & 1;
        if (!mbar_wait(&q_empty[qb], ((il >> 1) & 1) ^ 1u, args.status, abort_flag)) return false;
        const Item it = item_at(il);
        const int row0 = it.b * S;
        mbar_arrive_expect_tx(&q_full[qb], it.valid1 ? 2 * kQBytes : kQBytes);
        tma_load_2d(smem + Smem::q + (2 * qb) * kQBytes, &tmQ, &q_full[qb], it.h * kDh, row0 + it.q0);
        if (it.valid1)
          tma_load_2d(smem + Smem::q + (2 * qb + 1) * kQBytes, &tmQ, &q_full[qb], it.h * kDh, row0 + it.q0 + kQ);
        const int bit = 2 * kStages + qb;
        pending |= 1u << bit;
        pending_par = (pending_par & ~(1u << bit)) | (static_cast<uint32_t>((il >> 1) & 1) << bit);
        return true;
      };
      bool ok = load_q(0);
      int uk = 0, uv = 0;
      while (ok && uv < total_u) {
        // K runs up to kStages tiles ahead of V, so a group's next scores never wait for P V
        const bool take_k = uk < total_u && uk < uv + kStages;
        const int u = take_k ? uk : uv;
        const int st = u % kStages;
        const uint32_t ph = (u / kStages) & 1;
        uint64_t* empty = take_k ? &k_empty[st] : &v_empty[st];
        uint64_t* full = take_k ? &k_full[st] : &v_full[st];
        if (!mbar_wait(empty, ph ^ 1u, args.status, abort_flag)) break;
        const int il = u / nkv;
        const int j = u % nkv;
        const Item it = item_at(il);
        mbar_arrive_expect_tx(full, kKVBytes);
        tma_load_2d(smem + (take_k ? Smem::k : Smem::v) + st * kKVBytes, &tmKV, full,
                    (take_k ? H : 2 * H) + it.h * kDh, it.b * S + j * kKV);
        const int bit = st + (take_k ? 0 : kStages);
        pending |= 1u << bit;
        pending_par = (pending_par & ~(1u << bit)) | (ph << bit);
        if (take_k) {
          ++uk;
          // the next item's Q once this item's keys are all on their way
          if (j == nkv - 1 && il + 1 < my_items && !load_q(il + 1)) break;
        } else {
          ++uv;
        }
      }
      if (*abort_flag) {  // let in-flight copies land before the CTA exits
        for (int bit = 0; bit < 2 * kStages + 2; ++bit) {
          if (!(pending & (1u << bit))) continue;
          uint64_t* full = bit < kStages ? &k_full[bit]
                                         : (bit < 2 * kStages ? &v_full[bit - kStages] : &q_full[bit - 2 * kStages]);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(full, (pending_par >> bit) & 1u) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t q_addr = smem_u32(smem + Smem::q);
      const uint32_t k_addr = smem_u32(smem + Smem::k);
      const uint32_t v_addr = smem_u32(smem + Smem::v);
      const uint32_t p_addr = smem_u32(smem + Smem::p);
      int ns[2] = {0, 0};    // S issued per group
      int npv[2] = {0, 0};   // P V issued per group
      int nit[2] = {0, 0};   // items started (first P V) per group
      bool ok = true;
      // S_u of group w = Q[w] K_u^T into S[w][ns % 2]
      auto issue_s = [&](int u, int w) -> bool {
        const int il = u / nkv, j = u % nkv;
        const Item it = item_at(il);
        const bool last_w = (w == 1) || !it.valid1;
        if (w == 1 && !it.valid1) return true;
        const int st = u % kStages;
        if (!mbar_wait(&k_full[st], (u / kStages) & 1, args.status, abort_flag)) return false;
        if (!mbar_wait(&q_full[il & 1], (il >> 1) & 1, args.status, abort_flag)) return false;
        const int sb = ns[w] & 1;
        if (!mbar_wait(&s_empty[2 * w + sb], ((ns[w] >> 1) & 1) ^ 1u, args.status, abort_flag)) return false;
        tc_fence_after();
        const uint32_t qa = q_addr + ((il & 1) * 2 + w) * kQBytes;
#pragma unroll
        for (int k = 0; k < kDh / 16; ++k) {
          const uint64_t ad = sdesc_sw128(qa + k * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_addr + st * kKVBytes + k * 32, 16, 1024);
          umma_bf16_ss(tmem + 128 * w + 64 * sb, ad, bd, kIdescS, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[2 * w + sb]);
        if (last_w) {
          umma_commit(&k_empty[st]);
          if (j == nkv - 1) umma_commit(&q_empty[il & 1]);
        }
        ++ns[w];
        return true;
      };
      // O[w][item % 2] (+)= P_u V_u
      auto issue_pv = [&](int u, int w) -> bool {
        const int il = u / nkv, j = u % nkv;
        const Item it = item_at(il);
        if (w == 1 && !it.valid1) return true;
        const bool last_w = (w == 1) || !it.valid1;
        const int st = u % kStages;
        const int pb = npv[w] & 1;
        const int ob = nit[w] & 1;
        if (j == 0 && !mbar_wait(&o_empty[2 * w + ob], ((nit[w] >> 1) & 1) ^ 1u, args.status, abort_flag))
          return false;
        if (!mbar_wait(&p_full[2 * w + pb], (npv[w] >> 1) & 1, args.status, abort_flag)) return false;
        if (!mbar_wait(&v_full[st], (u / kStages) & 1, args.status, abort_flag)) return false;
        tc_fence_after();
        const uint32_t pa = p_addr + (2 * w + pb) * kPBytes;
#pragma unroll
        for (int k = 0; k < kKV / 16; ++k) {
          const uint64_t ad = sdesc_sw128(pa + k * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(v_addr + st * kKVBytes + k * 2048, 8192, 1024);
          umma_bf16_ss(tmem + kTmemO + 128 * w + 64 * ob, ad, bd, kIdescPV, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&p_empty[2 * w + pb]);
        if (last_w) umma_commit(&v_empty[st]);
        if (j == nkv - 1) {
          umma_commit(&o_full[2 * w + ob]);
          ++nit[w];
        }
        ++npv[w];
        return true;
      };
      for (int u = 0; ok && u < 2 && u < total_u; ++u)
        for (int w = 0; ok && w < 2; ++w) ok = issue_s(u, w);
      for (int u = 0; ok && u < total_u; ++u) {
        for (int w = 0; ok && w < 2; ++w) {
          ok = issue_pv(u, w);
          if (ok && u + 2 < total_u) ok = issue_s(u + 2, w);
        }
      }
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kIntraKernelTimeoutNs) {
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax groups
    const int w = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the group's tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float sl2 = args.scale_log2;
    int t = 0;   // this group's tile count (S / P buffers)
    int io = 0;  // this group's item count (O buffers)
    bool ok = true;
    for (int il = 0; ok && il < my_items; ++il) {
      const Item it = item_at(il);
      if (w == 1 && !it.valid1) continue;
      const int ob = io & 1;
      const uint32_t o_col = kTmemO + 128 * w + 64 * ob;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < nkv; ++j, ++t) {
        const int sb = t & 1;
        const uint32_t sph = (t >> 1) & 1;
        if (!mbar_wait(&s_full[2 * w + sb], sph, args.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[2][32];
        tmem_ld32(tmem + lane_off + 128 * w + 64 * sb, sr[0]);
        tmem_ld32(tmem + lane_off + 128 * w + 64 * sb + 32, sr[1]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[2 * w + sb]);
        const int kbase = j * kKV;
        if (kbase + kKV > S) {
#pragma unroll
          for (int c = 0; c < kKV; ++c)
            if (kbase + c >= S) sr[c >> 5][c & 31] = 0xff800000u;
        }
#define SV(c) __uint_as_float(sr[(c) >> 5][(c) & 31])
        float pm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = SV(i);
#pragma unroll
        for (int c = 8; c < kKV; ++c) pm[c & 7] = fmaxf(pm[c & 7], SV(c));
        const float tmx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                                fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))) * sl2;
        if (j == 0) {
          m = tmx;  // key 0 of the sequence is always valid, so m is finite
        } else if (__any_sync(0xffffffffu, tmx > m + kRescaleThreshold)) {
          // raise this warp's reference maxima; O holds this item's earlier tiles once the
          // group's previous P V (tile t - 1) has completed
          const float mn = fmaxf(m, tmx);
          const float alpha = ex2_approx(m - mn);
          m = mn;
          l *= alpha;
          const int tp = t - 1;
          if (!__all_sync(0xffffffffu,
                          mbar_wait(&p_empty[2 * w + (tp & 1)], (tp >> 1) & 1, args.status, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int hh = 0; hh < 4; ++hh) {
            uint32_t o[16];
            tmem_ld16(tmem + lane_off + o_col + 16 * hh, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st16(tmem + lane_off + o_col + 16 * hh, o);
          }
          tmem_wait_st();
        }
        // P_t -> smem P[w][sb] (A operand of P V, 128-byte swizzle), once P V of tile t - 2
        // has read that buffer
        if (!mbar_wait(&p_empty[2 * w + sb], sph ^ 1u, args.status, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* prow = smem + Smem::p + (2 * w + sb) * kPBytes + (r >> 3) * 1024 + (r & 7) * 128;
        float rsp[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t wd[4];
          float ps = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p0 = ex2_approx(fmaf(SV(8 * c + 2 * e), sl2, -m));
            const float p1 = ex2_approx(fmaf(SV(8 * c + 2 * e + 1), sl2, -m));
            ps += p0 + p1;
            wd[e] = pack_bf16x2(p0, p1);
          }
          rsp[c] = ps;
          *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
#undef SV
        l += ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) + ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7]));
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[2 * w + sb]);
      }
      if (!ok) break;
      // ---- this item's output rows: O / l -> bf16, and the log-sum-exp
      if (!mbar_wait(&o_full[2 * w + ob], (io >> 1) & 1, args.status, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int q = it.q0 + w * kQ + r;
      const float inv = 1.f / l;
      uint4* dst = reinterpret_cast<uint4*>(args.out + (static_cast<long long>(it.b) * S + q) * H + it.h * kDh);
#pragma unroll 1
      for (int hh = 0; hh < 4; ++hh) {
        uint32_t o0[16];
        tmem_ld16(tmem + lane_off + o_col + 16 * hh, o0);
        tmem_wait_ld();
        if (q < S) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(o0[8 * c + e]) * inv;
            dst[2 * hh + c] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                         pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
          }
        }
      }
      if (q < S)
        args.lse[(static_cast<long long>(it.b) * args.heads + it.h) * S + q] = (m + log2f(l)) * 0.69314718055994531f;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[2 * w + ob]);
      ++io;
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

void attn_fwd_persistent(const torch::Tensor& qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t S,
                         int64_t heads) {
  using namespace fa;
  check_cuda_bf16(qkv, "qkv");
  check_cuda_bf16(out, "out");
  check_cuda_f32(lse, "lse");
  const int64_t H = heads * kDh;
  REVPP_CHECK(qkv.is_contiguous() && qkv.size(0) == B * S && qkv.size(1) == 3 * H, "qkv must be [B*S, 3H]");
  REVPP_CHECK(out.is_contiguous() && out.size(0) == B * S && out.size(1) == H, "out must be [B*S, H]");
  REVPP_CHECK(lse.numel() >= B * heads * S, "lse too small");
  REVPP_CHECK(S >= 1 && B >= 1 && heads >= 1, "empty attention problem");
  c10::cuda::CUDAGuard guard(qkv.device());
  const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  const CUtensorMap tq = make_tmap_2d(qkv.data_ptr(), bf, 2, 3 * H, B * S, 3 * H * 2, 64, kQ, sw);
  const CUtensorMap tkv = make_tmap_2d(qkv.data_ptr(), bf, 2, 3 * H, B * S, 3 * H * 2, 64, kKV, sw);
  Args a;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.S = static_cast<int>(S);
  a.heads = static_cast<int>(heads);
  a.npairs = static_cast<int>((S + 2 * kQ - 1) / (2 * kQ));
  a.num_items = static_cast<int>(a.npairs * heads * B);
  a.nkv = static_cast<int>((S + kKV - 1) / kKV);
  a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(kDh)));
  a.status = status_device_ptr();
  constexpr int smem = Smem::total + 1024;
  static int configured_for = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_for != dev) {
    REVPP_CUDA_CHECK(
        cudaFuncSetAttribute(attn_fwd_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured_for = dev;
  }
  const int grid = std::max(1, std::min(a.num_items, num_sms()));
  attn_fwd_persistent_kernel<<<grid, kThreads, smem, cur_stream()>>>(tq, tkv, a);
  REVPP_CHECK_LAUNCH();
}

}  // namespace revpp
