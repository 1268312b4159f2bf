// Flash attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
// Head dim 64; same interface and numerics as attn_fwd in attention.cu (qkv packed as
// nn.MultiheadAttention's in_proj output, o [B*S, H] bf16, lse [B, heads, S] fp32).
//
// One CTA per (query tile of 128 rows, head, sequence); 64-key tiles.  Two softmax
// warpgroups split the key tiles of the CTA: group w takes tiles j with j % 2 == w, with
// its own TMEM scores S[w], output accumulator O[w], P tile, running maximum and sum, so
// the groups never wait for each other until the end, where they exchange maxima and sums
// and each merges half of the output columns (O = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / l).
// The softmax is issue-bound, not MUFU-bound (moving a quarter of the exponentials to an
// FP32-pipe polynomial made it slower): the scale / shift and the row sums run as packed
// fp32 pairs (FFMA2 / FADD2) and the row maximum as three-input maxima.  Sixteen softmax warps
// per SM (two CTAs) keep the exp / max / pack work of one group running while the other
// waits on the tensor core.
//   warp 0     : TMA producer - Q once, then K_j / V_j into a 3-deep ring (no multicast)
//   warp 1     : TMEM allocator and MMA issuer (one thread):
//                  S_j    = Q K_j^T   (M 128, N 64, K 64)  -> TMEM S[j % 2]
//                  O[j%2] += P_j V_j  (M 128, N 64, K 64)
//                S_{j+1} is issued before waiting for P_j.
//   warps 2-5  : softmax group 0 (even key tiles); warps 6-9: group 1 (odd key tiles);
//                one thread per query row: S row from TMEM, P_j = exp2(S * scale - m) as
//                bf16 into a 128-byte-swizzled smem tile (the MMA's A operand).
// Each group keeps a reference maximum m that is raised only when a tile's maximum
// exceeds it by more than 8 (log2 units): P stays <= 256, and the rescale of O (through
// tcgen05.ld / st, after the group's previous P V has landed) is rare.  Softmax is
// invariant to the reference maximum, so this equals the exact-max formulation up to
// rounding.
// Shared memory ~98 KB and 256 TMEM columns, so two CTAs share an SM.
#include "common.cuh"
#include "host.h"

namespace revpp {

namespace {
constexpr int kQ = 128;      // query rows per CTA
constexpr int kKV = 64;      // keys per tile
constexpr int kDh = 64;      // head dim
constexpr int kStages = 3;   // K/V ring depth
constexpr int kThreads = 320;
constexpr uint32_t kQBytes = kQ * kDh * 2;     // 16 KB
constexpr uint32_t kKVBytes = kKV * kDh * 2;   // 8 KB (one of K or V)
constexpr uint32_t kPBytes = kQ * kKV * 2;     // 16 KB
constexpr uint32_t kTmemCols = 256;            // S[2] (64 each) + O[2] (64 each)
constexpr uint32_t kTmemO = 128;
constexpr float kRescaleThreshold = 8.0f;      // log2 units: P <= 2^8
// The kernel's template argument PACKED: 1 = packed fp32 pairs and three-input maxima in the
// softmax, 0 = scalar (kept for comparison, REVPP_ATTN_PACKED=0).
constexpr uint32_t kIdescS = idesc_bf16(kQ, kKV, false, false);
constexpr uint32_t kIdescPV = idesc_bf16(kQ, kDh, false, true);

struct SmemLayout {
  // offsets from the 1024-aligned base
  static constexpr uint32_t q = 0;
  static constexpr uint32_t k = q + kQBytes;                      // kStages x 8 KB
  static constexpr uint32_t v = k + kStages * kKVBytes;           // kStages x 8 KB
  static constexpr uint32_t p = v + kStages * kKVBytes;           // 2 x 16 KB (one per group)
  static constexpr uint32_t stats = p + 2 * kPBytes;              // m, l per row of each group
  static constexpr uint32_t bars = stats + 4 * kQ * 4;
  static constexpr uint32_t total = bars + 256;
};
}  // namespace

struct AttnTcArgs {
  __nv_bfloat16* out;
  float* lse;
  int S, heads;
  float scale_log2;
  int* status;
  // optional [grid][32] globaltimer stamps of the CTA's phases (measurement aid)
  unsigned long long* phase_ns = nullptr;
};

constexpr int kPhaseSlots = 32;  // per CTA: 8 phases, then per-tile events of the first 4 tiles
__device__ __forceinline__ void phase_stamp(unsigned long long* ph, int k) {
  if (ph != nullptr) {
    const long long cta = blockIdx.x + static_cast<long long>(gridDim.x) * (blockIdx.y + static_cast<long long>(gridDim.y) * blockIdx.z);
    ph[cta * kPhaseSlots + k] = globaltimer_ns();
  }
}

template <int PACKED>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                       const AttnTcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SmemLayout::bars);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;               // [kStages]
  uint64_t* k_empty = k_full + kStages;     // [kStages] freed by S_j
  uint64_t* v_full = k_empty + kStages;     // [kStages]
  uint64_t* v_empty = v_full + kStages;     // [kStages] freed by P_j V_j
  uint64_t* s_full = v_empty + kStages;     // [2] per group
  uint64_t* s_empty = s_full + 2;           // [2]
  uint64_t* p_full = s_empty + 2;           // [2]
  uint64_t* p_empty = p_full + 2;           // [2]
  uint64_t* pv_done = p_empty + 2;          // [2] once per P V of the group (in order)
  uint64_t* comb = pv_done + 2;             // [2] group w's m, l are in shared memory
  uint64_t* drain = comb + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_stat = reinterpret_cast<float*>(smem + SmemLayout::stats);  // [m0, l0, m1, l1][kQ]

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
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_empty[i], 1);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(&comb[0], 4);
    mbar_init(&comb[1], 4);
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
  pdl_wait();  // barrier and TMEM set-up overlapped the previous kernel's tail
  pdl_trigger();
  if (threadIdx.x == 0) phase_stamp(args.phase_ns, 0);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      mbar_arrive_expect_tx(q_full, kQBytes);
      tma_load_2d(smem + SmemLayout::q, &tmQ, q_full, h * kDh, row0 + q0);
      // K_j as soon as S_{j-3} has read its stage, V_j once P_{j-3} V_{j-3} has: keys run
      // ahead of values, so the scores of a group's next tile never wait for P V
      uint32_t issued = 0, issued_par = 0;  // bits 0..2: K stages, 3..5: V stages
      int jk = 0, jv = 0;
      while (jv < nkv) {
        const bool take_k = jk < nkv && jk < jv + kStages;
        const int j = take_k ? jk : jv;
        const int st = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        uint64_t* empty = take_k ? &k_empty[st] : &v_empty[st];
        uint64_t* full = take_k ? &k_full[st] : &v_full[st];
        if (!mbar_wait(empty, ph ^ 1u, args.status, abort_flag)) break;
        mbar_arrive_expect_tx(full, kKVBytes);
        tma_load_2d(smem + (take_k ? SmemLayout::k : SmemLayout::v) + st * kKVBytes, &tmKV, full,
                    (take_k ? H : 2 * H) + h * kDh, row0 + j * kKV);
        const int bit = st + (take_k ? 0 : kStages);
        issued |= 1u << bit;
        issued_par = (issued_par & ~(1u << bit)) | (ph << bit);
        if (take_k) {
          ++jk;
        } else {
          ++jv;
        }
      }
      if (*abort_flag) {
        // let in-flight copies land before the CTA exits
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
        for (int bit = 0; bit < 2 * kStages; ++bit) {
          if (!(issued & (1u << bit))) continue;
          uint64_t* full = bit < kStages ? &k_full[bit] : &v_full[bit - kStages];
          const uint64_t t1 = globaltimer_ns();
          while (!mbar_try_wait(full, (issued_par >> bit) & 1u) && globaltimer_ns() - t1 < 100000000ull) {
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
      // S_j = Q K_j^T into S[j % 2], once group j % 2 has read S_{j-2}
      auto issue_s = [&](int j) -> bool {
        const int st = j % kStages;
        const int w = j & 1;
        if (!mbar_wait(&k_full[st], (j / kStages) & 1, args.status, abort_flag)) return false;
        if (j == 0) phase_stamp(args.phase_ns, 1);  // Q and the first K have landed
        if (!mbar_wait(&s_empty[w], ((j >> 1) & 1) ^ 1u, args.status, abort_flag)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kDh / 16; ++k) {
          const uint64_t ad = sdesc_sw128(q_addr + k * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_addr + st * kKVBytes + k * 32, 16, 1024);
          umma_bf16_ss(tmem + w * kKV, ad, bd, kIdescS, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[w]);
        umma_commit(&k_empty[st]);
        return true;
      };
      // O[j % 2] += P_j V_j, once group j % 2 has stored P_j (and any rescale of O)
      auto issue_pv = [&](int j) -> bool {
        const int w = j & 1;
        const int st = j % kStages;
        if (!mbar_wait(&p_full[w], (j >> 1) & 1, args.status, abort_flag)) return false;
        if (!mbar_wait(&v_full[st], (j / kStages) & 1, args.status, abort_flag)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kKV / 16; ++k) {
          const uint64_t ad = sdesc_sw128(p_addr + w * kPBytes + k * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(v_addr + st * kKVBytes + k * 2048, 8192, 1024);
          umma_bf16_ss(tmem + kTmemO + w * kDh, ad, bd, kIdescPV, (j >= 2 || k > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[w]);
        umma_commit(&p_empty[w]);
        umma_commit(&v_empty[st]);
        return true;
      };
      // scores run two tiles ahead of P V: S_{j+2} (the same group's next tile) is issued
      // as soon as that group has read S_j, before waiting for its P_j
      for (int j = 0; ok && j < 2 && j < nkv; ++j) ok = issue_s(j);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + 2 < nkv && !issue_s(j + 2)) {
          ok = false;
          break;
        }
        if (!issue_pv(j)) {
          ok = false;
          break;
        }
      }
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kIntraKernelTimeoutNs) {
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax groups
    const int w = (warp - 2) >> 2;               // group: key tiles j with j % 2 == w
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;           // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t o_col = kTmemO + w * kDh;
    uint8_t* prow = smem + SmemLayout::p + w * kPBytes + (r >> 3) * 1024 + (r & 7) * 128;
    float m = -INFINITY, l = 0.f;
    const float sl2 = args.scale_log2;
    bool ok = true;
    int t = 0;  // this group's tile count
    for (int j = w; j < nkv; j += 2, ++t) {
      const uint32_t par = t & 1;
      if (!mbar_wait(&s_full[w], par, args.status, abort_flag)) {
        ok = false;
        break;
      }
      if (t == 0 && warp == 2 && lane == 0) phase_stamp(args.phase_ns, 2);  // first scores ready
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld32(tmem + lane_off + w * kKV, sr[0]);
      tmem_ld32(tmem + lane_off + w * kKV + 32, sr[1]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[w]);
      // raw scores (the softmax scale, > 0, is applied after the max, folded into one FMA);
      // keys past the sequence end read as -inf
      const int kbase = j * kKV;
      if (kbase + kKV > S) {
#pragma unroll
        for (int c = 0; c < kKV; ++c)
          if (kbase + c >= S) sr[c >> 5][c & 31] = 0xff800000u;
      }
#define SV(c) __uint_as_float(sr[(c) >> 5][(c) & 31])
      // row max as 8 independent chains
      float pm[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pm[i] = SV(i);
      float tmx;
      if constexpr (PACKED) {
#pragma unroll
        for (int c = 8; c + 16 <= kKV; c += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) pm[i] = max3f(pm[i], SV(c + i), SV(c + 8 + i));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = fmaxf(pm[i], SV(kKV - 8 + i));
        tmx = max3f(max3f(pm[0], pm[1], pm[2]), max3f(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7])) * sl2;
      } else {
#pragma unroll
        for (int c = 8; c < kKV; ++c) pm[c & 7] = fmaxf(pm[c & 7], SV(c));
        tmx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                    fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))) * sl2;
      }
      if (t == 0) {
        m = tmx;  // key 0 of every tile is below S, so m is finite
      } else if (__any_sync(0xffffffffu, tmx > m + kRescaleThreshold)) {
        // raise the reference maximum of this warp's rows; O[w] holds this group's earlier
        // tiles once its previous P V has completed
        const float mn = fmaxf(m, tmx);
        const float alpha = ex2_approx(m - mn);
        m = mn;
        l *= alpha;
        if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[w], (t - 1) & 1, args.status, abort_flag))) {
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
      // P_j -> smem (A operand of P V, 128-byte swizzle: 16-byte chunk c of row r at c ^ (r & 7))
      if (!mbar_wait(&p_empty[w], par ^ 1u, args.status, abort_flag)) {
        ok = false;
        break;
      }
      if constexpr (PACKED) {
        // x = s * scale - m and the row sums on packed pairs; four pair accumulators
        const uint64_t sc2 = f32x2(sl2, sl2), nm2 = f32x2(-m, -m);
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};  // +0.0f pairs
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t wd[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float x0, x1;
            f32x2_split(fma_f32x2(f32x2(SV(8 * c + 2 * e), SV(8 * c + 2 * e + 1)), sc2, nm2), x0, x1);
            const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
            acc[e] = add_f32x2(acc[e], f32x2(p0, p1));
            wd[e] = pack_bf16x2(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
        float a0, a1;
        f32x2_split(add_f32x2(add_f32x2(acc[0], acc[1]), add_f32x2(acc[2], acc[3])), a0, a1);
        l += a0 + a1;
      } else {
        float rsp[8];  // row-sum partials, one per 16-byte unit
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
        l += ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) + ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7]));
      }
#undef SV
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[w]);
    }
    if (warp == 2 && lane == 0) phase_stamp(args.phase_ns, 3);  // group 0's last P handed over
    // this group's last P V has landed in O[w]
    bool fin = ok;
    if (fin && t > 0) fin = mbar_wait(&pv_done[w], (t - 1) & 1, args.status, abort_flag);
    // both groups publish their maximum and sum (m = -inf, l = 0 without key tiles); then
    // each merges and stores half of the output row: group w takes columns 32w .. 32w + 31
    s_stat[(2 * w) * kQ + r] = fin ? m : -INFINITY;
    s_stat[(2 * w + 1) * kQ + r] = fin ? l : 0.f;
    __syncwarp();
    if (lane == 0) mbar_arrive(&comb[w]);
    fin = fin && mbar_wait(&comb[w ^ 1], 0, args.status, abort_flag);
    if (warp == 2 && lane == 0) phase_stamp(args.phase_ns, 4);  // merge starts
    if (__all_sync(0xffffffffu, fin)) {
      tc_fence_after();
      const float m0 = s_stat[r], l0 = s_stat[kQ + r];
      const float m1 = s_stat[2 * kQ + r], l1 = s_stat[3 * kQ + r];
      const float mx = fmaxf(m0, m1);
      const float a0 = ex2_approx(m0 - mx);  // group 0 always has key tiles: m0 is finite
      const float a1 = l1 > 0.f ? ex2_approx(m1 - mx) : 0.f;
      const float lt = l0 * a0 + l1 * a1;
      const float inv = 1.f / lt;
      const float c0 = a0 * inv, c1 = a1 * inv;
      const bool two = nkv >= 2;  // group 1 has key tiles (uniform over the CTA)
      const int q = q0 + r;
      uint4* dst = reinterpret_cast<uint4*>(args.out + (static_cast<long long>(row0) + q) * H + h * kDh + 32 * w);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t col = 32 * w + 16 * hh;
        uint32_t o0[16], o1[16];
        tmem_ld16(tmem + lane_off + kTmemO + col, o0);
        if (two) tmem_ld16(tmem + lane_off + kTmemO + kDh + col, o1);
        tmem_wait_ld();
        if (q < S) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float x1 = two ? __uint_as_float(o1[8 * c + e]) * c1 : 0.f;
              f[e] = fmaf(__uint_as_float(o0[8 * c + e]), c0, x1);
            }
            dst[2 * hh + c] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                         pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
          }
        }
      }
      if (w == 0 && q < S)
        args.lse[(static_cast<long long>(b) * args.heads + h) * S + q] = (mx + log2f(lt)) * 0.69314718055994531f;
      if (warp == 2 && lane == 0) phase_stamp(args.phase_ns, 5);  // merge and stores issued
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) phase_stamp(args.phase_ns, 6);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

void attn_fwd_tc(const torch::Tensor& qkv, torch::Tensor out, torch::Tensor lse, int64_t B, int64_t S,
                 int64_t heads, const c10::optional<torch::Tensor>& phase_ns) {
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
  if (phase_ns.has_value() && phase_ns->defined()) {
    REVPP_CHECK(phase_ns->scalar_type() == at::kLong && phase_ns->is_cuda() && phase_ns->is_contiguous() &&
                    phase_ns->numel() >= ((S + kQ - 1) / kQ) * heads * B * kPhaseSlots,
                "phase_ns must be a CUDA int64 tensor of grid x 32 entries");
    a.phase_ns = reinterpret_cast<unsigned long long*>(phase_ns->data_ptr());
  }
  constexpr int smem = SmemLayout::total + 1024;
  static const bool packed = [] {
    const char* e = std::getenv("REVPP_ATTN_PACKED");
    return e == nullptr || std::atoi(e) != 0;
  }();
  auto kern = packed ? attn_fwd_tc_kernel<1> : attn_fwd_tc_kernel<0>;
  static int configured_for = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_for != dev) {
    for (auto k : {attn_fwd_tc_kernel<0>, attn_fwd_tc_kernel<1>})
      REVPP_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured_for = dev;
  }
  dim3 grid(static_cast<unsigned>((S + kQ - 1) / kQ), static_cast<unsigned>(heads), static_cast<unsigned>(B));
  launch_pdl(kern, grid, dim3(kThreads), smem, cur_stream(), tq, tkv, a);
  REVPP_CHECK_LAUNCH();
}


// ====================================================================== backward
// Flash attention backward on tcgen05.  Persistent: one CTA per SM takes the work items
// (key tile of 128, head, sequence) blockIdx.x, blockIdx.x + gridDim.x, ...; for each it
// walks the query tiles (128 queries each):
//   S^T  = K Q_j^T      (M 128 keys, N 128 queries, K 64)   -> TMEM cols [0, 128)
//   dP^T = V dO_j^T     (same shape)                         -> TMEM cols [128, 256)
//   softmax warps (one thread per key): P^T = exp(S^T * scale - lse_q) as bf16 pairs into
//       TMEM cols [448, 512), dS^T = P^T * (dP^T - D_q) as bf16 into a 128-byte-swizzled
//       smem tile
//   dV  += P^T dO_j     (M 128 keys, N 64, K 128 queries; A = P^T from TMEM)
//                                                            -> TMEM cols [256, 320)
//   dK  += dS^T Q_j     (same)                               -> TMEM cols [320, 384)
//   dQ_j = dS K         (M 128 queries, N 64, K 128 keys; dS read MN-major from the dS^T
//                        tile)                               -> TMEM cols [384, 448)
//   dQ warps (one thread per query) stage dQ_j * scale in shared memory and add each
//       256-byte row to an fp32 buffer with a bulk reduction (performed in L2).
// Warps: 0 TMA producer, 1 MMA issuer, 2-5 softmax (queries 0-31) / final dK, 6-9 dQ,
// 10-13 softmax (queries 32-63) / final dV, 14-17 and
// 18-21 softmax (queries 64-95, 96-127): four warps per scheduler share the exp / dS work
// (with two, the per-tile softmax was latency-bound).
// Overlap: as soon as the softmax of tile j has consumed S^T / dP^T, the issuer starts
// S^T / dP^T of tile j+1 (if its Q / dO rows have landed; else after this tile's MMAs) and
// then the dV / dK / dQ MMAs of tile j, so the softmax of tile j+1 runs while the tensor
// core works on tile j.  dS^T is therefore double-buffered
// in shared memory; P^T (one TMEM buffer) is rewritten only after the previous tile's dV
// MMAs have read it.
// Between items: the next item's first Q / dO tile loads while the current item ends, its K /
// V once the current item's MMAs have completed, and its first S^T / dP^T (TMEM [0, 256))
// runs while the dK / dV warps read the finished dK / dV out of TMEM [256, 384) and store
// them, so set-up and write-out of an item overlap the neighbouring items' work instead of
// leaving the SM idle (barrier and TMEM set-up happen once per CTA).
namespace {
constexpr int kBK = 128;  // keys per work item
constexpr int kBQ = 128;  // queries per tile
constexpr int kBwdGroups = 4;                  // softmax groups, kQG queries of a tile each
constexpr int kQG = 128 / kBwdGroups;
constexpr int kBwdThreads = 64 + 128 + 32 * 4 * kBwdGroups;  // producer, MMA, dQ warps, softmax groups
constexpr uint32_t kTile = 128 * 64 * 2;       // 16 KB: a [128 x 64] bf16 tile
constexpr uint32_t kSqTile = 2 * kTile;        // 32 KB: a [128 x 128] bf16 tile (2 swizzle chunks)
constexpr uint32_t kDqStride = 272;  // 256-byte dQ rows padded by 16: row r's chunk k is in bank group (r + k) % 8
struct BwdSmem {
  static constexpr uint32_t k = 0;
  static constexpr uint32_t v = k + kTile;
  static constexpr uint32_t q = v + kTile;              // 2 buffers
  static constexpr uint32_t dout = q + 2 * kTile;       // 2 buffers
  static constexpr uint32_t dst = dout + 2 * kTile;     // dS^T, 2 buffers
  static constexpr uint32_t stats = dst + 2 * kSqTile;  // per softmax warp: lse*log2e [kQG], D [kQG]
  static constexpr uint32_t dq = stats + 4 * kBwdGroups * 2 * kQG * 4;  // dQ_j fp32, 128 rows of 64, 272-byte stride
  static constexpr uint32_t red = dq + 128 * kDqStride;   // dK / dV column sums: 4 quarters x 128
  static constexpr uint32_t bars = red + 4 * 128 * 4;
  static constexpr uint32_t total = bars + 256;
};
static_assert(BwdSmem::total + 1024 <= 232448, "attention backward exceeds the shared-memory limit");
static_assert(8 * 4096 <= kSqTile, "the dK / dV staging tiles must fit in one dS^T buffer");
constexpr uint32_t kIdescSq = idesc_bf16(128, 128, false, false);
constexpr uint32_t kIdescKD = idesc_bf16(128, 64, false, true);
constexpr uint32_t kIdescQD = idesc_bf16(128, 64, true, true);
constexpr uint32_t kTmemPt = 448;  // P^T as bf16 pairs: 128 queries in 64 columns

}  // namespace

struct AttnBwdTcArgs {
  const float* lse;   // [B, heads, S]
  const float* D;     // [B, heads, S]
  float* dq_acc;      // [B*S, H] fp32, zeroed
  __nv_bfloat16* dqkv;
  int S, heads, B;
  float scale, scale_log2;
  int* status;
  float* colsum = nullptr;  // [3H] fp32 or null: += column sums of the bf16 dK / dV written here
  unsigned long long* phase_ns = nullptr;  // optional [grid][32] globaltimer stamps (measurement aid)
};

// Column sums over the 32 rows (lanes) of a warp: v holds this lane's 32 columns; returns
// the sum of column `lane` (recursive halving: 31 shuffles instead of 32 x 5).
__device__ __forceinline__ float warp_column_sums32(float (&v)[32], int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool up = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = up ? v[i] : v[i + w];
      const float keep = up ? v[i + w] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return v[0];
}

template <int PACKED>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmDO,
                       const AttnBwdTcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + BwdSmem::bars);
  uint64_t* kv_full = bar + 0;
  uint64_t* q_full = bar + 1;     // [2]
  uint64_t* q_empty = bar + 3;    // [2]
  uint64_t* s_full = bar + 5;
  uint64_t* p_full = bar + 6;
  uint64_t* p_empty = bar + 7;    // [2] (P^T / dS^T buffers)
  uint64_t* dq_full = bar + 9;
  uint64_t* dq_empty = bar + 10;
  uint64_t* kv_done = bar + 11;
  uint64_t* drain = bar + 12;
  uint64_t* grp_bar = bar + 13;   // the eight softmax warps' own barrier (bounded waits)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* cs_bar = bar + 16;    // the eight dK / dV warps' column sums are in shared memory
  uint64_t* pt_free = bar + 17;   // the dV MMAs of a tile have read P^T from TMEM
  uint64_t* s_free = bar + 22;    // the eight softmax warps have read S^T / dP^T of a tile
  float* s_stats = reinterpret_cast<float*>(smem + BwdSmem::stats);  // [softmax warp][2 kQG]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = args.S;
  const int H = args.heads * 64;
  const int nq = (S + kBQ - 1) / kBQ;
  const int nkt = (S + kBK - 1) / kBK;
  // persistent: work item it = (key tile, head, sequence), key tile fastest; the CTA takes
  // items blockIdx.x, blockIdx.x + gridDim.x, ...  Barrier phases follow the CTA's running
  // counts: g = query tiles so far, n = items so far.
  const int n_items = nkt * args.heads * args.B;
  auto item_kt = [&](int it) { return it % nkt; };
  auto item_h = [&](int it) { return (it / nkt) % args.heads; };
  auto item_b = [&](int it) { return it / (nkt * args.heads); };
  // phase stamps (measurement aid) describe the CTA's first item; slot 7 is the CTA's end
  auto stamp = [&](int n, int slot) {
    if (n == 0) phase_stamp(args.phase_ns, slot);
  };

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 4 * kBwdGroups);
    mbar_init(&p_empty[0], 1);
    mbar_init(&p_empty[1], 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    mbar_init(kv_done, 1);
    mbar_init(drain, 1);
    mbar_init(grp_bar, 8);
    mbar_init(cs_bar, 8);
    mbar_init(pt_free, 1);
    mbar_init(s_free, 4 * kBwdGroups);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQKV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // barrier and TMEM set-up overlapped the previous kernel's tail
  pdl_trigger();
  if (threadIdx.x == 0) phase_stamp(args.phase_ns, 0);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      // The query tiles of each item into the two-deep Q / dO ring; after an item's first
      // tile (whose buffer frees a tile before the previous item ends), its K / V, once every
      // MMA of the previous item has completed (kv_done)
      uint32_t kv_issued = 0, issued = 0, issued_par = 0;
      uint32_t g = 0;
      int n = 0;
      bool ok = true;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++n) {
        const int h = item_h(it);
        const int row0 = item_b(it) * S;
        for (int j = 0; j < nq; ++j, ++g) {
          const int bb = g & 1;
          const uint32_t par = (g >> 1) & 1;
          if (!mbar_wait(&q_empty[bb], par ^ 1u, args.status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&q_full[bb], 2 * kTile);
          tma_load_2d(smem + BwdSmem::q + bb * kTile, &tmQKV, &q_full[bb], h * 64, row0 + j * kBQ);
          tma_load_2d(smem + BwdSmem::dout + bb * kTile, &tmDO, &q_full[bb], h * 64, row0 + j * kBQ);
          issued |= 1u << bb;
          issued_par = (issued_par & ~(1u << bb)) | (par << bb);
          if (j == 0) {
            if (n > 0 && !mbar_wait(kv_done, (n - 1) & 1, args.status, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(kv_full, 2 * kTile);
            tma_load_2d(smem + BwdSmem::k, &tmQKV, kv_full, H + h * 64, row0 + item_kt(it) * kBK);
            tma_load_2d(smem + BwdSmem::v, &tmQKV, kv_full, 2 * H + h * 64, row0 + item_kt(it) * kBK);
            ++kv_issued;
          }
        }
      }
      if (*abort_flag) {
        // let this CTA's copies in flight land before it exits
        if (kv_issued > 0) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(kv_full, (kv_issued - 1) & 1) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
        for (int s = 0; s < 2; ++s) {
          if (!(issued & (1u << s))) continue;
          const uint64_t t1 = globaltimer_ns();
          while (!mbar_try_wait(&q_full[s], (issued_par >> s) & 1u) && globaltimer_ns() - t1 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t a_k = smem_u32(smem + BwdSmem::k);
      const uint32_t a_v = smem_u32(smem + BwdSmem::v);
      const uint32_t a_q = smem_u32(smem + BwdSmem::q);
      const uint32_t a_do = smem_u32(smem + BwdSmem::dout);
      const uint32_t a_ds = smem_u32(smem + BwdSmem::dst);
      // S^T_j = K Q_j^T and dP^T_j = V dO_j^T into TMEM [0, 256)
      auto issue_s = [&](int j) {
        const int bb = j & 1;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          umma_bf16_ss(tmem, sdesc_sw128(a_k + k * 32, 16, 1024), sdesc_sw128(a_q + bb * kTile + k * 32, 16, 1024),
                       kIdescSq, k > 0);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          umma_bf16_ss(tmem + 128, sdesc_sw128(a_v + k * 32, 16, 1024),
                       sdesc_sw128(a_do + bb * kTile + k * 32, 16, 1024), kIdescSq, k > 0);
        }
        umma_commit(s_full);
      };
      uint32_t g = 0;  // query tiles so far (all of this CTA's items)
      int n = 0;
      bool ok = true;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++n) {
        // K / V of this item; S^T / dP^T of its first tile (the softmax warps have read the
        // previous tile's, and dK / dV of the previous item live in other TMEM columns)
        if (!mbar_wait(kv_full, n & 1, args.status, abort_flag) ||
            !mbar_wait(&q_full[g & 1], (g >> 1) & 1, args.status, abort_flag))
          break;
        stamp(n, 1);  // K, V and the first Q / dO have landed
        tc_fence_after();
        issue_s(g);
        for (int j = 0; j < nq; ++j, ++g) {
          const int bb = g & 1;
          const uint32_t jp = g & 1;
          const uint32_t pb = g & 1;
          // the softmax warps have read S^T / dP^T of tile g from TMEM: start tile g+1 now,
          // so its scores are computed while they finish tile g and its softmax overlaps
          // this tile's gradient MMAs
          if (!mbar_wait(s_free, jp, args.status, abort_flag)) {
            ok = false;
            break;
          }
          if (j < 4) stamp(n, 8 + 4 * j + 2);  // tile j's scores read
          tc_fence_after();
          // S of tile g+1 goes first if its Q / dO rows have landed; otherwise this tile's
          // gradient MMAs go first, so they (and the release of this tile's Q / dO buffer,
          // which the load of tile g+2 waits for) never wait on the load of tile g+1
          bool s_next = false;
          if (j + 1 < nq && mbar_try_wait(&q_full[(g + 1) & 1], ((g + 1) >> 1) & 1)) {
            tc_fence_after();
            issue_s(g + 1);
            s_next = true;
          }
          // softmax of tile g is done: P^T of tile g is in TMEM, dS^T in buffer pb.  For the
          // item's first tile this also orders the dV / dK MMAs below (accumulate = 0) after
          // the previous item's dK / dV were read out: the dK / dV warps drain before they
          // take part in this tile's softmax
          if (!mbar_wait(p_full, jp, args.status, abort_flag)) {
            ok = false;
            break;
          }
          if (j < 4) stamp(n, 8 + 4 * j + 3);  // tile j's gradient MMAs issued
          tc_fence_after();
          const uint32_t a_dsj = a_ds + pb * kSqTile;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            // dV += P^T dO   (A = P^T from TMEM, 16 queries = 8 columns per MMA; B = dO,
            // MN-major: d contiguous, queries as K rows)
            umma_bf16_ts(tmem + 256, tmem + kTmemPt + 8 * k, sdesc_sw128(a_do + bb * kTile + k * 2048, 8192, 1024),
                         kIdescKD, (j > 0 || k > 0));
          }
          umma_commit(pt_free);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t ka = (k >> 2) * kTile + (k & 3) * 32;   // K-major over queries (2 chunks)
            // dK += dS^T Q
            umma_bf16_ss(tmem + 320, sdesc_sw128(a_dsj + ka, 16, 1024),
                         sdesc_sw128(a_q + bb * kTile + k * 2048, 8192, 1024), kIdescKD, (j > 0 || k > 0));
          }
          // the dQ warps have read the previous tile's dQ from TMEM (dV / dK above need not wait)
          if (!mbar_wait(dq_empty, jp ^ 1u, args.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            // dQ = dS K : A = dS (queries contiguous in the dS^T tile -> MN-major, 64-query
            // chunks 16 KB apart), B = K (MN-major: d contiguous, keys as K rows)
            umma_bf16_ss(tmem + 384, sdesc_sw128(a_dsj + k * 2048, kTile, 1024),
                         sdesc_sw128(a_k + k * 2048, 8192, 1024), kIdescQD, k > 0);
          }
          umma_commit(dq_full);
          umma_commit(&p_empty[pb]);
          umma_commit(&q_empty[bb]);
          if (j + 1 < nq && !s_next) {
            if (!mbar_wait(&q_full[(g + 1) & 1], ((g + 1) >> 1) & 1, args.status, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(g + 1);
          }
        }
        if (!ok) break;
        // every MMA of this item has completed: K / V may be reloaded, dK / dV read out
        umma_commit(kv_done);
      }
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kIntraKernelTimeoutNs) {
      }
    }
  } else if (warp < 6 || warp >= 10) {
    // ------------------------------------------------------------------ softmax (keys)
    // kBwdGroups warpgroups: warps 2-5 take queries [0, kQG) of the tile, warps 10-13 the
    // next kQG, and so on; each warp owns the 32 TMEM lanes (keys) of its quarter.
    const int grp = warp < 6 ? 0 : (warp - 10) / 4 + 1;
    const int qb = grp * kQG;               // first query of this group within the tile
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;      // key row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* ds_base = smem + BwdSmem::dst;
    // Every softmax warp keeps its own copy of the LSE (log2 units; +inf past the sequence
    // end, so P = 0 there) and D of its group's kQG queries, fetched into registers one
    // tile ahead (lane l holds query qb + l): no warp waits for another's staging.
    float* wst = s_stats + (grp * 4 + quarter) * 2 * kQG;
    const float4* s_lse4 = reinterpret_cast<const float4*>(wst);
    const float4* s_D4 = reinterpret_cast<const float4*>(wst + kQG);
    auto fetch_stats = [&](int it, int t, float& l2, float& dd) {
      const long long bh = static_cast<long long>(item_b(it)) * args.heads + item_h(it);
      const int q = t * kBQ + qb + lane;
      l2 = q < S ? args.lse[bh * S + q] * 1.4426950408889634f : __int_as_float(0x7f800000);
      dd = q < S ? args.D[bh * S + q] : 0.f;
    };
    float nl2 = 0.f, ndd = 0.f;
    if (static_cast<int>(blockIdx.x) < n_items) fetch_stats(blockIdx.x, 0, nl2, ndd);
    bool ok = true;
    uint32_t g = 0;  // query tiles so far
    int n = 0;       // items so far
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++n) {
      const int k0 = item_kt(it) * kBK;
      const bool key_ok = k0 + r < S;
      for (int j = 0; j < nq; ++j, ++g) {
        const uint32_t jp = g & 1;
        const uint32_t pb = g & 1;
        __syncwarp();  // this warp's reads of the previous tile's stats are done
        wst[lane] = nl2;
        wst[kQG + lane] = ndd;
        __syncwarp();
        if (j + 1 < nq) {
          fetch_stats(it, j + 1, nl2, ndd);
        } else if (it + static_cast<int>(gridDim.x) < n_items) {
          fetch_stats(it + gridDim.x, 0, nl2, ndd);  // the next item's first tile
        }
        if (!mbar_wait(s_full, jp, args.status, abort_flag)) {
          ok = false;
          break;
        }
        if (j == 0 && warp == 2 && lane == 0) stamp(n, 2);  // first S^T / dP^T ready
        if (j < 4 && warp == 2 && lane == 0) stamp(n, 8 + 4 * j + 0);  // tile j: softmax starts
        tc_fence_after();
        const int sw = r & 7;
        // the dS^T tile is two 64-query swizzle chunks; this group's queries start at 16-byte
        // unit (qb % 64) / 8 of chunk qb / 64
        uint8_t* drow = ds_base + pb * kSqTile + (qb / 64) * kTile + (r >> 3) * 1024 + sw * 128;
        const int u0 = (qb % 64) / 8;
        const float sl2 = args.scale_log2;
        // kQG / 16 sub-chunks of 16 queries (latency is hidden by the other groups' warps)
        constexpr int KS = kQG / 16;
#pragma unroll
        for (int k = 0; k < KS; ++k) {
          uint32_t sv[16], dp[16];
          tmem_ld16(tmem + lane_off + qb + 16 * k, sv);
          tmem_ld16(tmem + lane_off + 128 + qb + 16 * k, dp);
          tmem_wait_ld();
          if (k == KS - 1) {  // every S^T / dP^T column of this tile is in registers
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
          }
          const int q4 = 4 * k;  // first float4 of this sub-chunk's LSE / D in the warp's copy
          uint32_t pw[8], dw[8];
          bool waited = true;
          if (key_ok && PACKED) {
            // the same on packed fp32 pairs: P = 2^(S * scale - lse), dS = bf16(P) (dP - D)
            const uint64_t sc2 = f32x2(sl2, sl2);
#pragma unroll
            for (int e4 = 0; e4 < 4; ++e4) {
              const float4 L = s_lse4[q4 + e4];
              const float4 Dq = s_D4[q4 + e4];
              float x0, x1, x2, x3;
              f32x2_split(fma_f32x2(f32x2(__uint_as_float(sv[4 * e4 + 0]), __uint_as_float(sv[4 * e4 + 1])), sc2,
                                    f32x2(-L.x, -L.y)), x0, x1);
              f32x2_split(fma_f32x2(f32x2(__uint_as_float(sv[4 * e4 + 2]), __uint_as_float(sv[4 * e4 + 3])), sc2,
                                    f32x2(-L.z, -L.w)), x2, x3);
              const uint32_t pp0 = pack_bf16x2(ex2_approx(x0), ex2_approx(x1));
              const uint32_t pp1 = pack_bf16x2(ex2_approx(x2), ex2_approx(x3));
              const float2 r0 = unpack_bf16x2(pp0), r1 = unpack_bf16x2(pp1);
              pw[2 * e4] = pp0;
              pw[2 * e4 + 1] = pp1;
              const uint64_t g0 = add_f32x2(f32x2(__uint_as_float(dp[4 * e4 + 0]), __uint_as_float(dp[4 * e4 + 1])),
                                            f32x2(-Dq.x, -Dq.y));
              const uint64_t g1 = add_f32x2(f32x2(__uint_as_float(dp[4 * e4 + 2]), __uint_as_float(dp[4 * e4 + 3])),
                                            f32x2(-Dq.z, -Dq.w));
              float d0, d1, d2, d3;
              f32x2_split(mul_f32x2(f32x2(r0.x, r0.y), g0), d0, d1);
              f32x2_split(mul_f32x2(f32x2(r1.x, r1.y), g1), d2, d3);
              dw[2 * e4] = pack_bf16x2(d0, d1);
              dw[2 * e4 + 1] = pack_bf16x2(d2, d3);
            }
          } else if (key_ok) {
#pragma unroll
            for (int e4 = 0; e4 < 4; ++e4) {
              const float4 L = s_lse4[q4 + e4];
              const float4 Dq = s_D4[q4 + e4];
              const float p0 = ex2_approx(fmaf(__uint_as_float(sv[4 * e4 + 0]), sl2, -L.x));
              const float p1 = ex2_approx(fmaf(__uint_as_float(sv[4 * e4 + 1]), sl2, -L.y));
              const float p2 = ex2_approx(fmaf(__uint_as_float(sv[4 * e4 + 2]), sl2, -L.z));
              const float p3 = ex2_approx(fmaf(__uint_as_float(sv[4 * e4 + 3]), sl2, -L.w));
              const uint32_t pp0 = pack_bf16x2(p0, p1), pp1 = pack_bf16x2(p2, p3);
              const float2 r0 = unpack_bf16x2(pp0), r1 = unpack_bf16x2(pp1);
              pw[2 * e4] = pp0;
              pw[2 * e4 + 1] = pp1;
              dw[2 * e4] = pack_bf16x2(r0.x * (__uint_as_float(dp[4 * e4 + 0]) - Dq.x),
                                       r0.y * (__uint_as_float(dp[4 * e4 + 1]) - Dq.y));
              dw[2 * e4 + 1] = pack_bf16x2(r1.x * (__uint_as_float(dp[4 * e4 + 2]) - Dq.z),
                                           r1.y * (__uint_as_float(dp[4 * e4 + 3]) - Dq.w));
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) pw[e] = dw[e] = 0u;
          }
          if (k == 0) {
            // only the stores wait: the dS^T buffer must have been read by the gradient MMAs of
            // tile g - 2, and P^T of the previous tile by its dV MMAs (warp-uniform: tcgen05.st
            // is a warp-wide instruction); the first sub-chunk's exponentials overlap those MMAs
            waited = mbar_wait(&p_empty[pb], ((g >> 1) & 1) ^ 1u, args.status, abort_flag);
            if (g > 0) waited = waited && mbar_wait(pt_free, (g - 1) & 1, args.status, abort_flag);
            waited = __all_sync(0xffffffffu, waited);
            tc_fence_after();
          }
          if (!waited) {
            ok = false;
            break;
          }
          // P^T: the 16 queries are TMEM columns kTmemPt + (qb + 16k) / 2 .. + 7 of this key's lane
          tmem_st8(tmem + lane_off + kTmemPt + qb / 2 + 8 * k, pw);
          // dS^T: 16 queries = 32 bytes = 16-byte units u0 + 2k, u0 + 2k + 1 of this row
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const uint32_t off = ((u0 + 2 * k + t) ^ sw) << 4;
            *reinterpret_cast<uint4*>(drow + off) = make_uint4(dw[4 * t], dw[4 * t + 1], dw[4 * t + 2], dw[4 * t + 3]);
          }
        }
        if (!ok) break;
        tmem_wait_st();
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        if (j < 4 && warp == 2 && lane == 0) stamp(n, 8 + 4 * j + 1);  // tile j: handed over
      }
      // final dK (group 0) and dV (group 1) for this warp's keys; the decision is made
      // warp-uniform since the column sums below shuffle across all lanes
      if (!ok) break;
      if (warp == 2 && lane == 0) stamp(n, 3);  // last tile's P^T / dS^T handed over
      // (groups 2 and up have no write-out).  The next item's first dV / dK MMAs wait for this
      // tile's successor's softmax, which these warps run only after the read-out below.
      if (grp < 2) {
        const bool fin = __all_sync(0xffffffffu, mbar_wait(kv_done, n & 1, args.status, abort_flag));
        if (warp == 2 && lane == 0) stamp(n, 4);  // dK / dV complete in TMEM
        if (!fin) {
          ok = false;
          break;
        }
        {
          const int h = item_h(it);
          const int row0 = item_b(it) * S;
          tc_fence_after();
          // The 64 columns of this warp's 32 key rows go through a 4 KB shared-memory tile
          // (rows of 128 bytes, 16-byte units XOR-swizzled by row) in the dS^T buffer of the
          // item's last tile, free once kv_done has fired (the next item's first tile writes the
          // other buffer, and its second tile only after these warps have read its first scores);
          // the warp then stores 4 rows x 128 contiguous bytes per instruction instead of one
          // 16-byte piece of 32 different rows.
          uint8_t* stg = smem + BwdSmem::dst + ((g - 1) & 1) * kSqTile + (grp * 4 + quarter) * 4096;
          float* red = reinterpret_cast<float*>(smem + BwdSmem::red);  // column sums
          // dK (TMEM cols 320..383, scaled) or dV (256..319), 32 columns per load
#pragma unroll 1
          for (int part = 2 * grp; part < 2 * grp + 2; ++part) {
            const bool is_k = part < 2;
            const int half = part & 1;
            uint32_t v[32];
            tmem_ld32(tmem + lane_off + (is_k ? 320 : 256) + 32 * half, v);
            tmem_wait_ld();
            const float sc = is_k ? args.scale : 1.f;
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
              pk[e] = pack_bf16x2(__uint_as_float(v[2 * e]) * sc, __uint_as_float(v[2 * e + 1]) * sc);
#pragma unroll
            for (int u = 0; u < 4; ++u)
              *reinterpret_cast<uint4*>(stg + lane * 128 + (((half * 4 + u) ^ (lane & 7)) << 4)) =
                  make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
            if (args.colsum != nullptr) {  // bias gradient of the K / V projections
              float cv[32];
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const float2 r2 = unpack_bf16x2(pk[e]);
                cv[2 * e] = key_ok ? r2.x : 0.f;
                cv[2 * e + 1] = key_ok ? r2.y : 0.f;
              }
              // this warp's 32 keys
              red[quarter * 128 + part * 32 + lane] = warp_column_sums32(cv, lane);
            }
          }
          __syncwarp();
          {
            const int u = lane & 7;
            const long long gcol = (grp == 0 ? H : 2 * H) + h * 64 + u * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int rr = 4 * i + (lane >> 3);  // key row within this warp's 32
              const int key = k0 + quarter * 32 + rr;
              if (key < S) {
                *reinterpret_cast<uint4*>(args.dqkv + (static_cast<long long>(row0) + key) * (3LL * H) + gcol) =
                    *reinterpret_cast<const uint4*>(stg + rr * 128 + ((u ^ (rr & 7)) << 4));
              }
            }
          }
          if (args.colsum != nullptr) {
            // One atomic per column and CTA: the 4 key quarters' sums are added here first (an
            // atomic per warp put 4 x (B * S / 128) same-address atomics in L2's queue per column).
            __syncwarp();
            if (lane == 0) mbar_arrive(cs_bar);
            if (grp == 0 && quarter == 0 && mbar_wait(cs_bar, n & 1, args.status, abort_flag)) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int c = i * 32 + lane;  // 0..63 dK columns, 64..127 dV columns
                const float sum = red[c] + red[128 + c] + red[256 + c] + red[384 + c];
                atomicAdd(args.colsum + (c < 64 ? H : 2 * H - 64) + h * 64 + c, sum);
              }
            }
          }
          if (warp == 2 && lane == 0) stamp(n, 5);  // dK written, column sums added
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ dQ (queries)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t g = 0;  // query tiles so far
    bool ok = true;
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
      const int h = item_h(it);
      const int row0 = item_b(it) * S;
      for (int j = 0; j < nq; ++j, ++g) {
        if (!mbar_wait(dq_full, g & 1, args.status, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t dq[2][32];
        tmem_ld32(tmem + lane_off + 384, dq[0]);
        tmem_ld32(tmem + lane_off + 416, dq[1]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_empty);
        // dQ_j * scale -> this query's 256-byte row of the staging tile, then one bulk
        // reduction per row into the fp32 accumulator (performed in L2; per-thread vector
        // atomics made the LSU queue and L2 the limit of this kernel's dQ path).
        const int q = j * kBQ + r;
        float* srow = reinterpret_cast<float*>(smem + BwdSmem::dq + r * kDqStride);
        bulk_wait_read_all();  // the previous tile's reduction has read this row
        const float sc = args.scale;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          reinterpret_cast<float4*>(srow)[k] =
              make_float4(__uint_as_float(dq[(4 * k) >> 5][(4 * k) & 31]) * sc,
                          __uint_as_float(dq[(4 * k + 1) >> 5][(4 * k + 1) & 31]) * sc,
                          __uint_as_float(dq[(4 * k + 2) >> 5][(4 * k + 2) & 31]) * sc,
                          __uint_as_float(dq[(4 * k + 3) >> 5][(4 * k + 3) & 31]) * sc);
        }
        fence_proxy_async_smem();
        if (q < S) {
          bulk_reduce_add_f32(args.dq_acc + (static_cast<long long>(row0) + q) * H + h * 64, srow, 256);
          bulk_commit_group();
        }
      }
      if (warp == 6 && lane == 0 && it == static_cast<int>(blockIdx.x)) phase_stamp(args.phase_ns, 6);
    }
    // the staging tile must outlive the reductions' reads; their writes to global memory
    // complete with the grid
    bulk_wait_read_all();
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) phase_stamp(args.phase_ns, 7);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// The backward kernel instance: packed fp32-pair softmax unless REVPP_ATTN_BWD_PACKED=0.
using AttnBwdKernel = void (*)(CUtensorMap, CUtensorMap, AttnBwdTcArgs);
static AttnBwdKernel attn_bwd_kernel() {
  static const bool packed = [] {
    const char* e = std::getenv("REVPP_ATTN_BWD_PACKED");
    return e == nullptr || std::atoi(e) != 0;
  }();
  return packed ? attn_bwd_tc_kernel<1> : attn_bwd_tc_kernel<0>;
}
// Persistent grid: one CTA per SM (shared memory allows one) that the GEMMs also use (the
// SMs reserved for NCCL stay free), at most one per work item.
static unsigned attn_bwd_grid(long long B, long long S, long long heads, int sms) {
  const long long items = ((S + kBK - 1) / kBK) * heads * B;
  return static_cast<unsigned>(std::max<long long>(1, std::min<long long>(items, sms)));
}
static cudaError_t attn_bwd_set_smem(int bytes) {
  for (AttnBwdKernel k : {attn_bwd_tc_kernel<0>, attn_bwd_tc_kernel<1>}) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

void attn_bwd_dot_launch(const torch::Tensor& dout, const torch::Tensor& out, torch::Tensor D, torch::Tensor dq_acc,
                         int64_t M, int64_t S, int64_t heads);
void attn_dq_convert_launch(const torch::Tensor& dq_acc, torch::Tensor dqkv, int64_t M, int64_t H);

// dqkv[:, 0:H] = bf16(dq_acc) and colsum[0:H] += column sums of those bf16 values.
__global__ void __launch_bounds__(256) attn_dq_convert_colsum_kernel(const float* __restrict__ dq_acc,
                                                                      __nv_bfloat16* __restrict__ dqkv, long long M,
                                                                      int H, float* __restrict__ colsum) {
  // Block (x, y) converts rows [r0, r1) of the 256 columns [256 y, 256 y + 256): 64 threads
  // per row (one 16-byte group each) x 4 rows, 16 loads in flight per thread.  The four
  // row-lanes' sums meet in shared memory, so each column gets one atomic per row block
  // (gridDim.x of them): a same-address atomic per 4-column group of every block of a
  // grid spanning all rows serialised in L2 and tripled this kernel's time.
  constexpr int U = 16;
  __shared__ float4 red[4][64];
  const int cg = threadIdx.x & 63;   // 4-column group within the slice
  const int rl = threadIdx.x >> 6;   // row lane 0..3
  const int c4 = blockIdx.y * 64 + cg;
  const long long rows_per = (M + gridDim.x - 1) / gridDim.x;
  const long long r0 = blockIdx.x * rows_per;
  const long long r1 = r0 + rows_per < M ? r0 + rows_per : M;
  const bool col_ok = 4 * c4 < H;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col_ok) {
    for (long long row = r0 + rl; row < r1; row += 4 * U) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long rr = row + 4LL * u;
        v[u] = rr < r1 ? __ldcs(reinterpret_cast<const float4*>(dq_acc + rr * H) + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long rr = row + 4LL * u;
        if (rr >= r1) break;
        const uint32_t p0 = pack_bf16x2(v[u].x, v[u].y), p1 = pack_bf16x2(v[u].z, v[u].w);
        *reinterpret_cast<uint2*>(dqkv + rr * 3LL * H + 4 * c4) = make_uint2(p0, p1);
        const float2 q0 = unpack_bf16x2(p0), q1 = unpack_bf16x2(p1);
        s.x += q0.x;
        s.y += q0.y;
        s.z += q1.x;
        s.w += q1.y;
      }
    }
  }
  red[rl][cg] = s;
  __syncthreads();
  if (rl == 0 && col_ok && r0 < r1) {
    const float4 a = red[0][cg], b = red[1][cg], c = red[2][cg], d = red[3][cg];
    atomicAdd(reinterpret_cast<float4*>(colsum + 4 * c4),
              make_float4(a.x + b.x + c.x + d.x, a.y + b.y + c.y + d.y, a.z + b.z + c.z + d.z, a.w + b.w + c.w + d.w));
  }
}

// colsum (optional, fp32 [3H]): += column sums of the bf16 dqkv, the q/k/v projection bias
// gradient, fused into the dK/dV write-out and the dQ conversion.
void attn_bwd_tc(const torch::Tensor& qkv, const torch::Tensor& out, const torch::Tensor& dout,
                 const torch::Tensor& lse, torch::Tensor dqkv, torch::Tensor dq_acc, torch::Tensor Dbuf, int64_t B,
                 int64_t S, int64_t heads, const c10::optional<torch::Tensor>& colsum,
                 const c10::optional<torch::Tensor>& phase_ns) {
  check_cuda_bf16(qkv, "qkv");
  check_cuda_bf16(out, "out");
  check_cuda_bf16(dout, "dout");
  check_cuda_bf16(dqkv, "dqkv");
  check_cuda_f32(lse, "lse");
  check_cuda_f32(dq_acc, "dq_acc");
  check_cuda_f32(Dbuf, "D");
  const int64_t H = heads * 64;
  const int64_t M = B * S;
  REVPP_CHECK(qkv.is_contiguous() && qkv.size(0) == M && qkv.size(1) == 3 * H, "qkv must be [B*S, 3H]");
  REVPP_CHECK(dqkv.is_contiguous() && dqkv.size(0) == M && dqkv.size(1) == 3 * H, "dqkv must be [B*S, 3H]");
  REVPP_CHECK(dout.is_contiguous() && dout.numel() == M * H && out.numel() == M * H, "out/dout must be [B*S, H]");
  REVPP_CHECK(dq_acc.numel() >= M * H && Dbuf.numel() >= B * heads * S, "scratch too small");
  c10::cuda::CUDAGuard guard(qkv.device());
  cudaStream_t st = cur_stream();
  attn_bwd_dot_launch(dout, out, Dbuf, dq_acc, M, S, heads);  // D, and dq_acc = 0
  const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  const CUtensorMap tq = make_tmap_2d(qkv.data_ptr(), bf, 2, 3 * H, M, 3 * H * 2, 64, 128, sw);
  const CUtensorMap tdo = make_tmap_2d(dout.data_ptr(), bf, 2, H, M, H * 2, 64, 128, sw);
  AttnBwdTcArgs a;
  a.lse = lse.data_ptr<float>();
  a.D = Dbuf.data_ptr<float>();
  a.dq_acc = dq_acc.data_ptr<float>();
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.S = static_cast<int>(S);
  a.heads = static_cast<int>(heads);
  a.B = static_cast<int>(B);
  a.scale = static_cast<float>(1.0 / std::sqrt(64.0));
  a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(64.0));
  a.status = status_device_ptr();
  float* cs = nullptr;
  if (colsum.has_value() && colsum->defined()) {
    check_cuda_f32(*colsum, "colsum");
    REVPP_CHECK(colsum->is_contiguous() && colsum->numel() >= 3 * H, "colsum must hold 3H floats");
    REVPP_CHECK((reinterpret_cast<uintptr_t>(colsum->data_ptr()) & 15) == 0,
                "colsum must be 16-byte aligned (vector atomics)");
    cs = colsum->data_ptr<float>();
  }
  a.colsum = cs;
  if (phase_ns.has_value() && phase_ns->defined()) {
    REVPP_CHECK(phase_ns->scalar_type() == at::kLong && phase_ns->is_cuda() && phase_ns->is_contiguous() &&
                    phase_ns->numel() >= ((S + kBK - 1) / kBK) * heads * B * kPhaseSlots,
                "phase_ns must be a CUDA int64 tensor of grid x 32 entries");
    a.phase_ns = reinterpret_cast<unsigned long long*>(phase_ns->data_ptr());
  }
  constexpr int smem = BwdSmem::total + 1024;
  static int configured_for = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_for != dev) {
    REVPP_CUDA_CHECK(attn_bwd_set_smem(smem));
    configured_for = dev;
  }
  launch_pdl(attn_bwd_kernel(), dim3(attn_bwd_grid(B, S, heads, gemm_grid_sms())), dim3(kBwdThreads), smem, st, tq,
             tdo, a);
  REVPP_CHECK_LAUNCH();
  if (cs == nullptr) {
    attn_dq_convert_launch(dq_acc, dqkv, M, H);
  } else {
    const unsigned slices = static_cast<unsigned>((H + 255) / 256);
    const unsigned row_blocks =
        static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(M / 64, num_sms() / slices)));
    attn_dq_convert_colsum_kernel<<<dim3(row_blocks, slices), 256, 0, st>>>(dq_acc.data_ptr<float>(),
                                                          reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), M,
                                                          static_cast<int>(H), cs);
    REVPP_CHECK_LAUNCH();
  }
}

}  // namespace revpp

// ------------------------------------------------------------------ allocation-free entry point
// Declared (and documented for users) in attention_noalloc.h.  It launches the same four
// steps as attn_bwd_tc above (zero dQ accumulator, D = rowsum(dO * O), the tcgen05
// backward kernel, dQ conversion) with its temporaries in the file-scope array below.
#include <mutex>

#include "attention_noalloc.h"

namespace revpp {

__global__ void attn_bwd_dot_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                    float* __restrict__ D, float* __restrict__ dq_acc, int M, int S, int heads);
__global__ void attn_dq_convert_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv, long long M,
                                       int H);

namespace {

// [0, 256): fallback status word; then the fp32 dQ accumulator; then D (256-byte aligned)
static __device__ __align__(256) unsigned char g_attn_bwd_scratch[REVPP_ATTN_BWD_NOALLOC_SCRATCH_BYTES];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_scratch_dev[kNoAllocMaxDevices] = {};

int noalloc_fail(int code, char* err, size_t errlen, const std::string& msg) {
  if (err != nullptr && errlen > 0) {
    const size_t n = std::min(errlen - 1, msg.size());
    std::memcpy(err, msg.data(), n);
    err[n] = '\0';
  }
  return code;
}

// Once per device, with that device current: the scratch array's device address and the
// backward kernel's dynamic shared-memory limit.
cudaError_t noalloc_setup(int dev, unsigned char** scratch) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_scratch_dev[dev] == nullptr) {
    unsigned char* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_attn_bwd_scratch);
    if (e != cudaSuccess) return e;
    e = attn_bwd_set_smem(BwdSmem::total + 1024);
    if (e != cudaSuccess) return e;
    g_noalloc_scratch_dev[dev] = p;
  }
  *scratch = g_noalloc_scratch_dev[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace revpp

extern "C" int revpp_attn_bwd_tc_noalloc(const void* qkv, const void* out, const void* dout, const float* lse,
                                         void* dqkv, int B, int S, int heads, int* status, void* stream, char* err,
                                         size_t errlen) {
  using namespace revpp;
  if (!qkv || !out || !dout || !lse || !dqkv || B <= 0 || S <= 0 || heads <= 0)
    return noalloc_fail(REVPP_NOALLOC_BAD_ARGUMENT, err, errlen, "null pointer or non-positive size");
  for (const void* p : {qkv, out, dout, static_cast<const void*>(lse), static_cast<const void*>(dqkv)})
    if (reinterpret_cast<uintptr_t>(p) & 15)
      return noalloc_fail(REVPP_NOALLOC_BAD_ARGUMENT, err, errlen, "every buffer must be 16-byte aligned");
  const long long H = 64LL * heads;
  const long long M = static_cast<long long>(B) * S;
  const unsigned long long dq_bytes = (static_cast<unsigned long long>(M * H) * 4ULL + 255ULL) & ~255ULL;
  const unsigned long long d_bytes = static_cast<unsigned long long>(M) * heads * 4ULL;
  const unsigned long long need = 256ULL + dq_bytes + d_bytes;
  if (need > REVPP_ATTN_BWD_NOALLOC_SCRATCH_BYTES)
    return noalloc_fail(REVPP_NOALLOC_TOO_LARGE, err, errlen,
                        "attention backward needs " + std::to_string(need) + " bytes of scratch for B=" +
                            std::to_string(B) + " S=" + std::to_string(S) + " heads=" + std::to_string(heads) +
                            "; the allocation-free entry point holds " +
                            std::to_string(REVPP_ATTN_BWD_NOALLOC_SCRATCH_BYTES) + " bytes");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
    return noalloc_fail(REVPP_NOALLOC_CUDA_ERROR, err, errlen, "no usable current CUDA device");
  unsigned char* scratch = nullptr;
  e = noalloc_setup(dev, &scratch);
  if (e != cudaSuccess)
    return noalloc_fail(REVPP_NOALLOC_CUDA_ERROR, err, errlen, std::string("set-up: ") + cudaGetErrorString(e));
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess)
    return noalloc_fail(REVPP_NOALLOC_CUDA_ERROR, err, errlen, std::string("SM count: ") + cudaGetErrorString(e));
  int* st_word = status ? status : reinterpret_cast<int*>(scratch);
  float* dq_acc = reinterpret_cast<float*>(scratch + 256);
  float* Dbuf = reinterpret_cast<float*>(scratch + 256 + dq_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  CUtensorMap tq, tdo;
  try {
    const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
    tq = make_tmap_2d(qkv, bf, 2, 3 * H, M, 3 * H * 2, 64, 128, sw);
    tdo = make_tmap_2d(dout, bf, 2, H, M, H * 2, 64, 128, sw);
  } catch (const std::exception& ex) {
    return noalloc_fail(REVPP_NOALLOC_BAD_ARGUMENT, err, errlen, ex.what());
  }
  {
    // D = rowsum(dO * O), and the dQ accumulator (which must start at zero) is cleared
    const long long threads = 256;
    const long long blocks = (M * heads * 8 + threads - 1) / threads;
    attn_bwd_dot_kernel<<<static_cast<unsigned>(blocks), static_cast<unsigned>(threads), 0, st>>>(
        static_cast<const __nv_bfloat16*>(dout), static_cast<const __nv_bfloat16*>(out), Dbuf, dq_acc,
        static_cast<int>(M), S, heads);
  }
  AttnBwdTcArgs a;
  a.lse = lse;
  a.D = Dbuf;
  a.dq_acc = dq_acc;
  a.dqkv = static_cast<__nv_bfloat16*>(dqkv);
  a.S = S;
  a.heads = heads;
  a.B = B;
  a.scale = static_cast<float>(1.0 / std::sqrt(64.0));
  a.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(64.0));
  a.status = st_word;
  attn_bwd_kernel()<<<attn_bwd_grid(B, S, heads, std::max(1, sms - sm_reserve())), kBwdThreads,
                      BwdSmem::total + 1024, st>>>(tq, tdo, a);
  {
    const long long n4 = M * H / 4;
    const long long threads = 256;
    attn_dq_convert_kernel<<<static_cast<unsigned>((n4 + threads - 1) / threads), static_cast<unsigned>(threads), 0,
                             st>>>(dq_acc, static_cast<__nv_bfloat16*>(dqkv), M, static_cast<int>(H));
  }
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return noalloc_fail(REVPP_NOALLOC_CUDA_ERROR, err, errlen, std::string("launch: ") + cudaGetErrorString(e));
  return REVPP_NOALLOC_OK;
}
