// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[M,N] (op)= A[M,K] * B[N,K]^T       bf16 operands, fp32 accumulation in TMEM
//
// Operands may be K-major (row-major [rows, K]) or MN-major (stored as [K, rows]);
// this covers forward (A K, B K), input-gradient (A K, B MN: the weight [N_out, K_in]
// read as [K_in rows] x [N_out reduction]) and weight-gradient (A MN, B MN: the
// activations [tokens, features] read along the token reduction) GEMMs without any
// transposed copies.
//
// Warp roles (320 threads):
//   warp 0      : TMA producer (one thread), STAGES-deep smem ring, no multicast
//   warp 1      : TMEM allocator + MMA issuer (one thread), tcgen05.mma 128xBNx16
//   warps 2..9  : epilogue, one (TMEM lane quarter, column half) each; TMEM ->
//                 registers (tcgen05.ld) -> fused op -> per-warp smem staging tile ->
//                 row-contiguous global stores
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue of
// tile i overlaps the main loop of tile i+1.
//
// Replaces the reference's cuBLAS GEMMs inside nn.Linear / nn.MultiheadAttention
// (BERT/models/bert_blocks.py:34-63) and their autograd backward.
#include <cstdlib>

#include "common.cuh"
#include "host.h"

namespace revpp {

enum GemmEpi : int {
  kEpiBF16 = 0,       // C_bf16 = bf16(acc + bias)
  kEpiGelu = 1,       // u = bf16(acc + bias); C_bf16 = bf16(gelu(u)); aux_out = u
  kEpiResid = 2,      // C_f32 = resid + sign * bf16(acc + bias)     (reversible coupling)
  kEpiAtomicF32 = 3,  // C_f32 += acc  (vector atomics; split-K and grad accumulation)
  kEpiDGelu = 4,      // C_bf16 = bf16(bf16(acc) * gelu'(aux))         (GELU backward)
  kEpiF32 = 5,        // C_f32 = acc + bias
  kEpiCount = 6,
};

struct GemmArgs {
  int M, N, K;
  int tiles_m, tiles_n, splits, kb_per_split, kb_total;
  void* C;
  long long ldc;
  const __nv_bfloat16* bias;  // [N] or null
  const __nv_bfloat16* aux;   // [M, ld_aux] bf16 (pre-activation for kEpiDGelu)
  __nv_bfloat16* aux_out;     // [M, ld_aux] bf16 (pre-activation written by kEpiGelu) or null
  long long ld_aux;
  const float* resid;  // [M, ld_resid] fp32 (kEpiResid)
  long long ld_resid;
  float sign;
  float* colsum_part;  // [ceil(M/32), N] fp32 or null: kEpiDGelu writes the column sums of every
                       // 32-row group of its (bf16) output there (reduced by gemm_colsum_reduce)
  int raster_m;        // 1: tiles numbered m-fastest (kept for measurements); 0: n-fastest
  int* status;
};

// Output tile of linear tile index t.  n-fastest (the default): the CTAs (pairs) of a
// persistent grid run consecutive tiles at the same time, so they share a few row blocks of
// A and all of B through L2, and A is read from DRAM about once.  m-fastest walks a whole
// column of tiles first: with many column tiles A is re-read from DRAM once per column.
struct TileCoord {
  int tm, tn, ts;
};
__device__ __forceinline__ TileCoord tile_coord(const GemmArgs& a, int t) {
  TileCoord c;
  if (a.raster_m) {
    c.tm = t % a.tiles_m;
    const int r = t / a.tiles_m;
    c.tn = r % a.tiles_n;
    c.ts = r / a.tiles_n;
  } else {
    c.tn = t % a.tiles_n;
    const int r = t / a.tiles_n;
    c.tm = r % a.tiles_m;
    c.ts = r / a.tiles_m;
  }
  return c;
}

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
// Epilogue warps EW = 8 or 16: warp w reads TMEM lane quarter (w % 4) and column group
// (w - 2) / 4 of the tile (EW / 4 groups).  The epilogue-heavy instances (GELU, GELU
// backward, residual) use 16 warps, four per scheduler, whose rounds are 32 columns so the
// registers fit 576 threads; the others 8 warps with 64-column bf16 rounds.
constexpr int kGemmEpiWarps = 8;  // default (plain epilogues)
template <int EW>
struct EpiGeom {
  static_assert(EW == 8 || EW == 16, "8 or 16 epilogue warps");
  static constexpr int kWarps = EW;
  static constexpr int kColGroups = EW / 4;
  static constexpr int kThreads = 64 + EW * 32;
};

// ------------------------------------------------------------------ epilogue
// Each epilogue warp owns 32 TMEM lanes (= 32 output rows) and a run of columns.  A
// tcgen05.ld gives every thread one row, so writing straight to global memory would make
// each warp-wide access touch 32 different rows.  Instead every round goes through a
// 4 KB per-warp staging tile (32 rows of up to 128 bytes, 16-byte units XOR-swizzled by
// row, which keeps both access patterns at the 4-wavefront minimum): threads write their
// row, then the warp moves (32 / NU) rows of NU contiguous 16-byte units per instruction,
// reading the residual / pre-activation inputs with the same row-contiguous pattern.
constexpr uint32_t kEpiStageBytes = 32 * 128;

__device__ __forceinline__ uint32_t epi_stg_off(int row, int unit) {
  return static_cast<uint32_t>(row * 128 + ((unit ^ (row & 7)) << 4));
}

template <int EPI, int EW = 8>
struct EpiTraits {
  static constexpr bool kBf16Stage = (EPI == kEpiBF16 || EPI == kEpiGelu || EPI == kEpiDGelu);
  static constexpr int kCols = (kBf16Stage && EW == 8) ? 64 : 32;  // output columns per staged round
  static constexpr int kElemPerUnit = kBf16Stage ? 8 : 4;
  static constexpr int kUnits = kCols / kElemPerUnit;  // 16-byte units per staged row: 4 or 8
  static constexpr int kRowsPerInst = 32 / kUnits;       // rows one warp instruction covers
  static constexpr int kIters = 32 / kRowsPerInst;       // warp instructions per round (= kUnits)
};

// Phase 1: this thread's row of the round (NU units) into the staging tile.
template <bool BF16, int NU>
__device__ __forceinline__ void epi_stage_row(uint8_t* stg, int lane, const float* v) {
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    uint4 w;
    if constexpr (BF16) {
      w = make_uint4(pack_bf16x2(v[8 * u + 0], v[8 * u + 1]), pack_bf16x2(v[8 * u + 2], v[8 * u + 3]),
                     pack_bf16x2(v[8 * u + 4], v[8 * u + 5]), pack_bf16x2(v[8 * u + 6], v[8 * u + 7]));
    } else {
      w = make_uint4(__float_as_uint(v[4 * u + 0]), __float_as_uint(v[4 * u + 1]), __float_as_uint(v[4 * u + 2]),
                     __float_as_uint(v[4 * u + 3]));
    }
    *reinterpret_cast<uint4*>(stg + epi_stg_off(lane, u)) = w;
  }
}

// Phase 2 for a plain copy of the staged tile (NU units per row) to a row-major output.
template <int ELEM_BYTES, int NU>
__device__ __forceinline__ void epi_copy_out(const uint8_t* stg, int lane, void* out, long long ld, int row0, int col0,
                                             int M, int N) {
  constexpr int E = 16 / ELEM_BYTES;
  constexpr int RPI = 32 / NU;
  const int u = lane % NU;
  const int col = col0 + u * E;
#pragma unroll
  for (int i = 0; i < NU; ++i) {
    const int rr = RPI * i + lane / NU;
    const uint4 w = *reinterpret_cast<const uint4*>(stg + epi_stg_off(rr, u));
    if (row0 + rr < M && col < N)
      *reinterpret_cast<uint4*>(static_cast<uint8_t*>(out) + ((static_cast<long long>(row0 + rr) * ld + col) * ELEM_BYTES)) = w;
  }
}

// Side input of an epilogue round (the fp32 residual of kEpiResid, the bf16 pre-activation
// of kEpiDGelu): kIters 16-byte units per lane, rows kRowsPerInst i + lane / kUnits, read
// row-contiguously like the stores.  With 8 epilogue warps it is loaded one round ahead of
// its use, so the latency of the global loads overlaps the previous round.
template <int EPI>
struct EpiSide {
  using T = uint4;
};
template <>
struct EpiSide<kEpiResid> {
  using T = float4;
};
template <int EPI>
__device__ __forceinline__ constexpr bool epi_has_side() {
  return EPI == kEpiResid || EPI == kEpiDGelu;
}

template <int EPI, int EW>
__device__ __forceinline__ void epi_load_side(const GemmArgs& a, int lane, int row0, int col0,
                                              typename EpiSide<EPI>::T (&sd)[EpiTraits<EPI, EW>::kIters]) {
  using T = EpiTraits<EPI, EW>;
  const int col = col0 + (lane % T::kUnits) * T::kElemPerUnit;
#pragma unroll
  for (int i = 0; i < T::kIters; ++i) {
    const int rr = T::kRowsPerInst * i + lane / T::kUnits;
    const bool ok = row0 + rr < a.M && col < a.N;
    if constexpr (EPI == kEpiResid) {
      sd[i] = ok ? *reinterpret_cast<const float4*>(a.resid + static_cast<long long>(row0 + rr) * a.ld_resid + col)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      sd[i] = ok ? *reinterpret_cast<const uint4*>(a.aux + static_cast<long long>(row0 + rr) * a.ld_aux + col)
                 : make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// L2 prefetch of the side input of a warp's next tile (rows row0 .. row0 + 31, columns
// col0 .. col0 + ncols): one 128-byte line per row and round, issued by the lane of that row,
// no registers held.  The register prefetch one round ahead then finds the lines in L2.
template <int EPI, int WARP_COLS>
__device__ __forceinline__ void epi_prefetch_side_l2(const GemmArgs& a, int lane, int row0, int col0) {
  const int row = row0 + lane;
  if (row >= a.M) return;
  constexpr int kRowBytes = WARP_COLS * (EPI == kEpiResid ? 4 : 2);
#pragma unroll
  for (int b = 0; b < kRowBytes / 128; ++b) {
    const int col = col0 + b * (EPI == kEpiResid ? 32 : 64);
    if (col >= a.N) break;
    const void* p = EPI == kEpiResid
                        ? static_cast<const void*>(a.resid + static_cast<long long>(row) * a.ld_resid + col)
                        : static_cast<const void*>(a.aux + static_cast<long long>(row) * a.ld_aux + col);
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
  }
}

// One staged round: `r` holds kCols accumulator columns of this thread's row
// (row0 + lane), starting at output column col0; `sd` the round's side input.
template <int EPI, int EW>
__device__ __forceinline__ void gemm_epilogue_round(const GemmArgs& a, uint8_t* stg, int lane, int row0, int col0,
                                                    const uint32_t* r,
                                                    const typename EpiSide<EPI>::T (&sd)[EpiTraits<EPI, EW>::kIters]) {
  using T = EpiTraits<EPI, EW>;
  constexpr int NC = T::kCols;
  constexpr int NU = T::kUnits;
  constexpr int RPI = T::kRowsPerInst;
  float v[NC];
#pragma unroll
  for (int j = 0; j < NC; ++j) v[j] = __uint_as_float(r[j]);
  if constexpr (EPI != kEpiDGelu && EPI != kEpiAtomicF32) {
    if (a.bias != nullptr) {
#pragma unroll
      for (int j = 0; j < NC / 8; ++j) {
        if (col0 + 8 * j < a.N) {
          const uint4 b = __ldg(reinterpret_cast<const uint4*>(a.bias + col0) + j);
          const float2 b0 = unpack_bf16x2(b.x), b1 = unpack_bf16x2(b.y), b2 = unpack_bf16x2(b.z),
                       b3 = unpack_bf16x2(b.w);
          v[8 * j + 0] += b0.x; v[8 * j + 1] += b0.y; v[8 * j + 2] += b1.x; v[8 * j + 3] += b1.y;
          v[8 * j + 4] += b2.x; v[8 * j + 5] += b2.y; v[8 * j + 6] += b3.x; v[8 * j + 7] += b3.y;
        }
      }
    }
  }
  const int u = lane % NU;
  const int col = col0 + u * T::kElemPerUnit;
  if constexpr (EPI == kEpiBF16 || EPI == kEpiF32) {
    epi_stage_row<T::kBf16Stage, NU>(stg, lane, v);
    __syncwarp();
    epi_copy_out<T::kBf16Stage ? 2 : 4, NU>(stg, lane, a.C, a.ldc, row0, col0, a.M, a.N);
  } else if constexpr (EPI == kEpiGelu) {
    // unit by unit, so the GELU values never coexist with all the accumulators; the bf16
    // pre-activations stay packed for the optional aux_out copy
    uint32_t pre[NC / 2];
#pragma unroll
    for (int uu = 0; uu < NU; ++uu) {
      uint32_t hw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float x0 = bf16r(v[8 * uu + 2 * e]), x1 = bf16r(v[8 * uu + 2 * e + 1]);
        pre[4 * uu + e] = pack_bf16x2(x0, x1);
        float y0, y1;
        gelu_erf2(x0, x1, y0, y1);
        hw[e] = pack_bf16x2(y0, y1);
      }
      *reinterpret_cast<uint4*>(stg + epi_stg_off(lane, uu)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
    __syncwarp();
    epi_copy_out<2, NU>(stg, lane, a.C, a.ldc, row0, col0, a.M, a.N);
    if (a.aux_out != nullptr) {
      __syncwarp();
#pragma unroll
      for (int uu = 0; uu < NU; ++uu)
        *reinterpret_cast<uint4*>(stg + epi_stg_off(lane, uu)) =
            make_uint4(pre[4 * uu], pre[4 * uu + 1], pre[4 * uu + 2], pre[4 * uu + 3]);
      __syncwarp();
      epi_copy_out<2, NU>(stg, lane, a.aux_out, a.ld_aux, row0, col0, a.M, a.N);
    }
  }
  else if constexpr (EPI == kEpiResid) {
    // C = resid + sign * bf16(acc + bias)
#pragma unroll
    for (int j = 0; j < NC; ++j) v[j] = bf16r(v[j]);
    epi_stage_row<false, NU>(stg, lane, v);
    __syncwarp();
    const float sg = a.sign;
#pragma unroll
    for (int i = 0; i < T::kIters; ++i) {
      const int rr = RPI * i + lane / NU;
      const uint4 w = *reinterpret_cast<const uint4*>(stg + epi_stg_off(rr, u));
      if (row0 + rr < a.M && col < a.N) {
        *reinterpret_cast<float4*>(static_cast<float*>(a.C) + static_cast<long long>(row0 + rr) * a.ldc + col) =
            make_float4(sd[i].x + sg * __uint_as_float(w.x), sd[i].y + sg * __uint_as_float(w.y),
                        sd[i].z + sg * __uint_as_float(w.z), sd[i].w + sg * __uint_as_float(w.w));
      }
    }
  } else if constexpr (EPI == kEpiDGelu) {
    // C = bf16(bf16(acc) * gelu'(aux)), aux = pre-activation; with colsum_part, the column
    // sums of this round's 32 rows go to row row0 / 32 of the partial-sum buffer
    epi_stage_row<true, NU>(stg, lane, v);
    __syncwarp();
    float cs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < T::kIters; ++i) {
      const int rr = RPI * i + lane / NU;
      const uint4 w = *reinterpret_cast<const uint4*>(stg + epi_stg_off(rr, u));
      if (row0 + rr < a.M && col < a.N) {
        const uint32_t wa[4] = {w.x, w.y, w.z, w.w};
        const uint32_t xa[4] = {sd[i].x, sd[i].y, sd[i].z, sd[i].w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 g = unpack_bf16x2(wa[e]);
          const float2 pre = unpack_bf16x2(xa[e]);
          float d0, d1;
          gelu_erf_grad2(pre.x, pre.y, d0, d1);
          float o0, o1;
          f32x2_split(mul_f32x2(f32x2(g.x, g.y), f32x2(d0, d1)), o0, o1);
          o[e] = pack_bf16x2(o0, o1);
          const float2 rs = unpack_bf16x2(o[e]);
          cs[2 * e] += rs.x;
          cs[2 * e + 1] += rs.y;
        }
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.C) + static_cast<long long>(row0 + rr) * a.ldc + col) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    if (a.colsum_part != nullptr) {  // warp-uniform
      // lanes with the same lane % NU hold the same 8 columns (different rows)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
#pragma unroll
        for (int m = NU; m < 32; m <<= 1) cs[e] += __shfl_xor_sync(0xffffffffu, cs[e], m);
      }
      if (lane < NU && row0 < a.M && col < a.N) {
        float* dst = a.colsum_part + static_cast<long long>(row0 >> 5) * a.N + col;
        *reinterpret_cast<float4*>(dst) = make_float4(cs[0], cs[1], cs[2], cs[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(cs[4], cs[5], cs[6], cs[7]);
      }
    }
  } else if constexpr (EPI == kEpiAtomicF32) {
    epi_stage_row<false, NU>(stg, lane, v);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < T::kIters; ++i) {
      const int rr = RPI * i + lane / NU;
      const uint4 w = *reinterpret_cast<const uint4*>(stg + epi_stg_off(rr, u));
      if (row0 + rr < a.M && col < a.N) {
        atomicAdd(reinterpret_cast<float4*>(static_cast<float*>(a.C) + static_cast<long long>(row0 + rr) * a.ldc + col),
                  make_float4(__uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z), __uint_as_float(w.w)));
      }
    }
  }
  __syncwarp();  // the staging tile is rewritten by the next round
}

// TMEM -> registers for one round (RC = 32 or 64 columns).
template <int RC>
__device__ __forceinline__ void epi_tmem_round(uint32_t taddr, uint32_t (&r)[RC]) {
  tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
  if constexpr (RC == 64) tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
  tmem_wait_ld();
}

// The epilogue of one warp for one tile: WARP_COLS accumulator columns starting at TMEM
// address `taddr` (lane quarter and column already applied), output rows row0..row0+31,
// output columns from col0.  With 8 epilogue warps, epilogues with a side input run two
// rounds per iteration with ping-pong side buffers, each loaded a round ahead; with 16
// the other warps of the scheduler hide the load, which is issued at the start of its round.
template <int EPI, int WARP_COLS, int EW>
__device__ __forceinline__ void gemm_epilogue_warp(const GemmArgs& a, uint8_t* stg, int lane, uint32_t taddr,
                                                   int row0, int col0, int next_row0 = -1, int next_col0 = 0) {
  using T = EpiTraits<EPI, EW>;
  constexpr int RC = T::kCols;
  constexpr int NI = T::kIters;
  using SideT = typename EpiSide<EPI>::T;
  if constexpr (epi_has_side<EPI>()) {
    if (next_row0 >= 0) epi_prefetch_side_l2<EPI, WARP_COLS>(a, lane, next_row0, next_col0);
  }
  if constexpr (epi_has_side<EPI>() && EW == 8) {
    SideT s0[NI], s1[NI];
    epi_load_side<EPI, EW>(a, lane, row0, col0, s0);
#pragma unroll 1
    for (int c = 0; c < WARP_COLS; c += 2 * RC) {
      if (col0 + c >= a.N) break;  // warp-uniform
      const bool more1 = c + RC < WARP_COLS && col0 + c + RC < a.N;
      if (more1) epi_load_side<EPI, EW>(a, lane, row0, col0 + c + RC, s1);
      uint32_t r[RC];
      epi_tmem_round<RC>(taddr + c, r);
      gemm_epilogue_round<EPI, EW>(a, stg, lane, row0, col0 + c, r, s0);
      if (!more1) break;
      if (c + 2 * RC < WARP_COLS && col0 + c + 2 * RC < a.N)
        epi_load_side<EPI, EW>(a, lane, row0, col0 + c + 2 * RC, s0);
      epi_tmem_round<RC>(taddr + c + RC, r);
      gemm_epilogue_round<EPI, EW>(a, stg, lane, row0, col0 + c + RC, r, s1);
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < WARP_COLS; c += RC) {
      if (col0 + c >= a.N) break;  // warp-uniform
      SideT sd[NI];
      if constexpr (epi_has_side<EPI>()) {
        epi_load_side<EPI, EW>(a, lane, row0, col0 + c, sd);
      } else {
#pragma unroll
        for (int i = 0; i < NI; ++i) sd[i] = SideT{};
      }
      uint32_t r[RC];
      epi_tmem_round<RC>(taddr + c, r);
      gemm_epilogue_round<EPI, EW>(a, stg, lane, row0, col0 + c, r, sd);
    }
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(EpiGeom<8>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs args) {
  constexpr int BM = kGemmBM, BK = kGemmBK;
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = BN * BK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = idesc_bf16(BM, BN, A_MN, B_MN);
  static_assert(BN % 64 == 0 && BN <= 256, "BN must be 64..256");
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM alloc must be a power of 2");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sEpi = smem + STAGES * STAGE_BYTES;  // EpiGeom<8>::kWarps x 4 KB staging tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + EpiGeom<8>::kWarps * kEpiStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&tfull[0], 1);
    mbar_init(&tfull[1], 1);
    mbar_init(&tempty[0], EpiGeom<8>::kWarps);
    mbar_init(&tempty[1], EpiGeom<8>::kWarps);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = args.tiles_m * args.tiles_n * args.splits;
  const int t_first = blockIdx.x, t_step = gridDim.x;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;  // per-stage bits, for the drain on abort
      for (int t = t_first; t < num_tiles; t += t_step) {
        const TileCoord tc = tile_coord(args, t);
        const int tm = tc.tm, tn = tc.tn;
        const int kb0 = tc.ts * args.kb_per_split;
        const int kb1 = min(args.kb_total, kb0 + args.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, args.status, abort_flag)) goto producer_abort;
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          if constexpr (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * BK, tm * BM);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_2d(a_dst + c * (BK * 128), &tmA, &full[stage], tm * BM + c * 64, kb * BK);
          }
          if constexpr (!B_MN) {
            tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, tn * BN);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(b_dst + c * (BK * 128), &tmB, &full[stage], tn * BN + c * 64, kb * BK);
          }
          issued |= (1u << stage);
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      goto producer_end;
    producer_abort:
      // Let every copy this thread issued land before the CTA leaves.
      for (int s = 0; s < STAGES; ++s) {
        if (issued & (1u << s)) {
          const uint32_t par = (issued_parity >> s) & 1u;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[s], par) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    producer_end:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      const uint32_t a_base = smem_u32(sA);
      const uint32_t b_base = smem_u32(sB);
      for (int t = t_first; t < num_tiles; t += t_step) {
        const int kb0 = tile_coord(args, t).ts * args.kb_per_split;
        const int kb1 = min(args.kb_total, kb0 + args.kb_per_split);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, args.status, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_s = a_base + stage * A_BYTES;
          const uint32_t b_s = b_base + stage * B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_s + k * 2048, BK * 128, 1024) : sdesc_sw128(a_s + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_s + k * 2048, BK * 128, 1024) : sdesc_sw128(b_s + k * 32, 16, 1024);
            umma_bf16_ss(d_tmem, ad, bd, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // All MMAs of this thread complete before TMEM is released.
      umma_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kIntraKernelTimeoutNs) {
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int ew = warp - 2;
    const int q = warp & 3;     // TMEM lane quarter this warp may access
    const int cg = ew >> 2;     // column half handled by this warp
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = t_first; t < num_tiles; t += t_step) {
      const TileCoord tc = tile_coord(args, t);
      if (!mbar_wait(&tfull[acc], acc_phase, args.status, abort_flag)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN + cg * (BN / EpiGeom<8>::kColGroups));
      int nrow = -1, ncol = 0;
      if (t + t_step < num_tiles) {
        const TileCoord nc = tile_coord(args, t + t_step);
        nrow = nc.tm * BM + q * 32;
        ncol = nc.tn * BN + cg * (BN / EpiGeom<8>::kColGroups);
      }
      gemm_epilogue_warp<EPI, BN / EpiGeom<8>::kColGroups, 8>(args, sEpi + ew * kEpiStageBytes, lane, taddr, tc.tm * BM + q * 32,
                                                   tc.tn * BN + cg * (BN / EpiGeom<8>::kColGroups), nrow, ncol);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ 2-SM variant
// A CTA pair (cluster of 2) computes a 256 x 256 tile with tcgen05.mma.cta_group::2:
// CTA r holds rows [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the
// B tile (the N half) in shared memory, and receives the 128 x 256 accumulator slice of
// its A rows in its own TMEM.  Each SM therefore moves 8 KB of operands per 128 x 256 x 16
// MMA step instead of 12 KB, which keeps the tensor pipe fed.
//   - both CTAs' TMA loads complete on the leader CTA's `full` barrier (the leader alone
//     posts the expected byte count); loads carry no multicast;
//   - the leader's single MMA thread issues the pair's MMAs and commits to `empty`, `tfull`
//     and `drain` in both CTAs with a multicast commit;
//   - the leader's `tempty` barrier counts the epilogue warps of both CTAs (the peer's
//     arrive remotely), so the accumulator is reused only after both halves are read.
template <int STAGES, bool A_MN, bool B_MN, int EPI, int EW>
__global__ void __launch_bounds__(EpiGeom<EW>::kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const GemmArgs args) {
  constexpr int BM = 128, BN = 256, BK = kGemmBK;  // per CTA: 128 A rows, 128 B rows; tile 256 x 256
  constexpr int HALF_N = BN / 2;
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = HALF_N * BK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = idesc_bf16(2 * BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sEpi = smem + STAGES * STAGE_BYTES;  // EpiGeom<EW>::kWarps x 4 KB staging tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + EpiGeom<EW>::kWarps * kEpiStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&tfull[0], 1);
    mbar_init(&tfull[1], 1);
    mbar_init(&tempty[0], 2 * EpiGeom<EW>::kWarps);
    mbar_init(&tempty[1], 2 * EpiGeom<EW>::kWarps);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc2(tmem_slot, TMEM_COLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();     // the set-up above overlapped the previous kernel's tail
  pdl_trigger();

  const int num_tiles = args.tiles_m * args.tiles_n * args.splits;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int t_first = cluster_id, t_step = num_clusters;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;
      const uint32_t full_leader0 = mapa_shared(smem_u32(&full[0]), 0);
      for (int t = t_first; t < num_tiles; t += t_step) {
        const TileCoord tc = tile_coord(args, t);
        const int tm = tc.tm, tn = tc.tn;
        const int kb0 = tc.ts * args.kb_per_split;
        const int kb1 = min(args.kb_total, kb0 + args.kb_per_split);
        const int a_row0 = tm * 2 * BM + crank * BM;
        const int b_row0 = tn * BN + crank * HALF_N;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, args.status, abort_flag)) goto producer_abort2;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
          const uint32_t fb = full_leader0 + stage * 8;
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          if constexpr (!A_MN) {
            tma_load_2d_2sm(a_dst, &tmA, fb, kb * BK, a_row0);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c) tma_load_2d_2sm(a_dst + c * (BK * 128), &tmA, fb, a_row0 + c * 64, kb * BK);
          }
          if constexpr (!B_MN) {
            tma_load_2d_2sm(b_dst, &tmB, fb, kb * BK, b_row0);
          } else {
#pragma unroll
            for (int c = 0; c < HALF_N / 64; ++c)
              tma_load_2d_2sm(b_dst + c * (BK * 128), &tmB, fb, b_row0 + c * 64, kb * BK);
          }
          issued |= (1u << stage);
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      goto producer_end2;
    producer_abort2:
      // let copies issued by this CTA land (their bytes are counted on the leader's barrier)
      for (int s = 0; s < STAGES; ++s) {
        if (leader && (issued & (1u << s))) {
          const uint32_t par = (issued_parity >> s) & 1u;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[s], par) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
      {
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {
        }
      }
    producer_end2:;
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (leader)
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      const uint32_t a_base = smem_u32(sA);
      const uint32_t b_base = smem_u32(sB);
      for (int t = t_first; t < num_tiles; t += t_step) {
        const int kb0 = tile_coord(args, t).ts * args.kb_per_split;
        const int kb1 = min(args.kb_total, kb0 + args.kb_per_split);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, args.status, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_s = a_base + stage * A_BYTES;
          const uint32_t b_s = b_base + stage * B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_s + k * 2048, BK * 128, 1024) : sdesc_sw128(a_s + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_s + k * 2048, BK * 128, 1024) : sdesc_sw128(b_s + k * 32, 16, 1024);
            umma2_bf16_ss(d_tmem, ad, bd, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma2_commit_mc(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma2_commit_mc(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      umma2_commit_mc(drain, 0x3);
    }
    if (lane == 0) {
      // both CTAs: every MMA writing this CTA's TMEM has completed before it is released
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kIntraKernelTimeoutNs) {
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int ew = warp - 2;
    const int q = warp & 3;
    const int cg = ew >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    for (int t = t_first; t < num_tiles; t += t_step) {
      const TileCoord tc = tile_coord(args, t);
      if (!mbar_wait(&tfull[acc], acc_phase, args.status, abort_flag)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN + cg * (BN / EpiGeom<EW>::kColGroups));
      int nrow = -1, ncol = 0;
      if (t + t_step < num_tiles) {
        const TileCoord nc = tile_coord(args, t + t_step);
        nrow = nc.tm * 2 * BM + crank * BM + q * 32;
        ncol = nc.tn * BN + cg * (BN / EpiGeom<EW>::kColGroups);
      }
      gemm_epilogue_warp<EPI, BN / EpiGeom<EW>::kColGroups, EW>(args, sEpi + ew * kEpiStageBytes, lane, taddr,
                                                   tc.tm * 2 * BM + crank * BM + q * 32,
                                                   tc.tn * BN + cg * (BN / EpiGeom<EW>::kColGroups), nrow, ncol);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, TMEM_COLS);
  }
  cluster_sync();
}

// colsum[n] += sum_r part[r, n] over the partial column sums of the GELU-backward epilogue.
// Block (x, y): 128 columns (a float4 per lane), rows y, y + gridDim.y, ... split over 8
// warps; one float4 atomic per lane and block row-group.
__global__ void __launch_bounds__(256) gemm_colsum_reduce_kernel(const float* __restrict__ part,
                                                                  float* __restrict__ colsum, int rows, int N) {
  __shared__ float4 red[8][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = blockIdx.x * 128 + lane * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col < N) {
    for (int r = blockIdx.y + gridDim.y * warp; r < rows; r += gridDim.y * 8) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(part + static_cast<long long>(r) * N + col));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && col < N) {
#pragma unroll
    for (int w = 1; w < 8; ++w) {
      const float4 v = red[w][lane];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    atomicAdd(reinterpret_cast<float4*>(colsum + col), acc);
  }
}

// ------------------------------------------------------------------ host side
namespace {

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
void launch_gemm_inst(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                      cudaStream_t st) {
  constexpr int smem = STAGES * (kGemmBM * kGemmBK * 2 + BN * kGemmBK * 2) + kGemmEpiWarps * kEpiStageBytes + 1024 + 256;
  auto kern = gemm_tc_kernel<BN, STAGES, A_MN, B_MN, EPI>;
  static int configured_for = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_for != dev) {
    REVPP_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured_for = dev;
  }
  kern<<<grid, EpiGeom<8>::kThreads, smem, st>>>(ta, tb, args);
  REVPP_CHECK_LAUNCH();
}

template <int STAGES, bool A_MN, bool B_MN, int EPI, int EW>
void launch_gemm2_inst(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                       cudaStream_t st) {
  constexpr int smem = STAGES * (kGemmBM * kGemmBK * 2 + 128 * kGemmBK * 2) + EW * kEpiStageBytes + 1024 + 256;
  auto kern = gemm_tc2_kernel<STAGES, A_MN, B_MN, EPI, EW>;
  static int configured_for = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_for != dev) {
    REVPP_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured_for = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(EpiGeom<EW>::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  REVPP_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, args));
  count_launch();
}

void dispatch_gemm2(bool a_mn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                    const GemmArgs& args, int grid, cudaStream_t st) {
  constexpr int ST = 6;   // 6 x 32 KB operand stages + 8 x 4 KB epilogue staging tiles
  constexpr int ST16 = 5;  // 5 x 32 KB operand stages + 16 x 4 KB epilogue staging tiles
  // 16 epilogue warps for the GELU epilogue and the residual epilogue of the K = 1024
  // GEMMs (measured at M = 32768: 257 -> 245 us, 92 -> 86 us); with K = 4096 the sixth
  // operand stage is worth more than the wider epilogue, and the GELU-backward epilogue
  // was slower on 16 warps (284 -> 290 us).  REVPP_GEMM_EPI_WARPS=8 keeps 8 everywhere.
  static const bool wide = [] {
    const char* e = std::getenv("REVPP_GEMM_EPI_WARPS");
    return e == nullptr || std::atoi(e) != 8;
  }();
  if (!a_mn && !b_mn) {
    switch (epi) {
      case kEpiBF16: return launch_gemm2_inst<ST, false, false, kEpiBF16, 8>(ta, tb, args, grid, st);
      case kEpiGelu:
        if (wide) return launch_gemm2_inst<ST16, false, false, kEpiGelu, 16>(ta, tb, args, grid, st);
        return launch_gemm2_inst<ST, false, false, kEpiGelu, 8>(ta, tb, args, grid, st);
      case kEpiResid:
        if (wide && args.K <= 1024)
          return launch_gemm2_inst<ST16, false, false, kEpiResid, 16>(ta, tb, args, grid, st);
        return launch_gemm2_inst<ST, false, false, kEpiResid, 8>(ta, tb, args, grid, st);
      case kEpiF32: return launch_gemm2_inst<ST, false, false, kEpiF32, 8>(ta, tb, args, grid, st);
      default: break;
    }
  } else if (!a_mn && b_mn) {
    switch (epi) {
      case kEpiBF16: return launch_gemm2_inst<ST, false, true, kEpiBF16, 8>(ta, tb, args, grid, st);
      case kEpiDGelu: return launch_gemm2_inst<ST, false, true, kEpiDGelu, 8>(ta, tb, args, grid, st);
      case kEpiF32: return launch_gemm2_inst<ST, false, true, kEpiF32, 8>(ta, tb, args, grid, st);
      default: break;
    }
  } else if (a_mn && b_mn) {
    if (epi == kEpiAtomicF32) return launch_gemm2_inst<ST, true, true, kEpiAtomicF32, 8>(ta, tb, args, grid, st);
  }
  REVPP_CHECK(false, "2-SM GEMM layout/epilogue combination not built: a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);
}

// Only the operand-layout / epilogue pairs the models use are instantiated:
//   A K-major, B K-major : forward GEMMs       (bf16, gelu, residual, f32)
//   A K-major, B MN-major: input-gradient GEMMs (bf16, gelu-backward, f32)
//   A MN-major, B MN-major: weight gradients   (atomic f32 accumulate)
void dispatch_gemm(bool a_mn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                   const GemmArgs& args, int grid, cudaStream_t st) {
  constexpr int BN = 256, ST = 4;  // 4 x 48 KB operand stages + 8 x 4 KB epilogue staging tiles
  if (!a_mn && !b_mn) {
    switch (epi) {
      case kEpiBF16: return launch_gemm_inst<BN, ST, false, false, kEpiBF16>(ta, tb, args, grid, st);
      case kEpiGelu: return launch_gemm_inst<BN, ST, false, false, kEpiGelu>(ta, tb, args, grid, st);
      case kEpiResid: return launch_gemm_inst<BN, ST, false, false, kEpiResid>(ta, tb, args, grid, st);
      case kEpiF32: return launch_gemm_inst<BN, ST, false, false, kEpiF32>(ta, tb, args, grid, st);
      default: break;
    }
  } else if (!a_mn && b_mn) {
    switch (epi) {
      case kEpiBF16: return launch_gemm_inst<BN, ST, false, true, kEpiBF16>(ta, tb, args, grid, st);
      case kEpiDGelu: return launch_gemm_inst<BN, ST, false, true, kEpiDGelu>(ta, tb, args, grid, st);
      case kEpiF32: return launch_gemm_inst<BN, ST, false, true, kEpiF32>(ta, tb, args, grid, st);
      default: break;
    }
  } else if (a_mn && b_mn) {
    if (epi == kEpiAtomicF32) return launch_gemm_inst<BN, ST, true, true, kEpiAtomicF32>(ta, tb, args, grid, st);
  }
  REVPP_CHECK(false, "GEMM layout/epilogue combination not built: a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);
}

}  // namespace

// A: if !a_mn, [M, K] row-major (row stride lda); if a_mn, [K, M] row-major.
// B: if !b_mn, [N, K] row-major; if b_mn, [K, N] row-major.
// variant: 0 = automatic (2-SM kernel unless M <= 128), 1 = one-CTA kernel, 2 = 2-SM kernel.
void gemm_tc(const torch::Tensor& A, bool a_mn, const torch::Tensor& B, bool b_mn, int64_t M, int64_t N, int64_t K,
             int64_t epi, torch::Tensor C, const c10::optional<torch::Tensor>& bias,
             const c10::optional<torch::Tensor>& aux, const c10::optional<torch::Tensor>& aux_out,
             const c10::optional<torch::Tensor>& resid, double sign, int64_t splits, int64_t variant,
             const c10::optional<torch::Tensor>& colsum) {
  check_cuda_bf16(A, "A");
  check_cuda_bf16(B, "B");
  REVPP_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm operands must be 2-D");
  REVPP_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm operands need unit inner stride");
  REVPP_CHECK(N % 32 == 0, "gemm N must be a multiple of 32, got ", N);
  REVPP_CHECK(M > 0 && N > 0 && K > 0, "gemm sizes must be positive");
  if (!a_mn) {
    REVPP_CHECK(A.size(0) >= M && A.size(1) >= K, "A shape mismatch");
  } else {
    REVPP_CHECK(A.size(0) >= K && A.size(1) >= M, "A (MN-major) shape mismatch");
  }
  if (!b_mn) {
    REVPP_CHECK(B.size(0) >= N && B.size(1) >= K, "B shape mismatch");
  } else {
    REVPP_CHECK(B.size(0) >= K && B.size(1) >= N, "B (MN-major) shape mismatch");
  }
  REVPP_CHECK(C.size(0) >= M && C.size(1) >= N, "C shape mismatch");
  const bool c_f32 = (epi == kEpiResid || epi == kEpiAtomicF32 || epi == kEpiF32);
  if (c_f32) {
    check_cuda_f32(C, "C");
  } else {
    check_cuda_bf16(C, "C");
  }
  REVPP_CHECK((C.stride(0) * (c_f32 ? 4 : 2)) % 16 == 0, "C row stride must be a multiple of 16 bytes");
  REVPP_CHECK(splits >= 1, "splits must be >= 1");
  REVPP_CHECK(splits == 1 || epi == kEpiAtomicF32, "split-K needs the atomic epilogue");
  c10::cuda::CUDAGuard guard(A.device());

  const bool two_sm = variant == 2 || (variant == 0 && M > kGemmBM);
  const int tile_m = two_sm ? 2 * kGemmBM : kGemmBM;
  GemmArgs args{};
  args.M = static_cast<int>(M);
  args.N = static_cast<int>(N);
  args.K = static_cast<int>(K);
  args.tiles_m = static_cast<int>((M + tile_m - 1) / tile_m);
  args.tiles_n = static_cast<int>((N + 255) / 256);
  args.kb_total = static_cast<int>((K + kGemmBK - 1) / kGemmBK);
  const int want_splits = static_cast<int>(std::min<int64_t>(splits, args.kb_total));
  args.kb_per_split = (args.kb_total + want_splits - 1) / want_splits;
  args.splits = (args.kb_total + args.kb_per_split - 1) / args.kb_per_split;
  args.C = C.data_ptr();
  args.ldc = C.stride(0);
  args.bias = nullptr;
  if (bias.has_value() && bias->defined()) {
    check_cuda_bf16(*bias, "bias");
    REVPP_CHECK(bias->numel() >= N && bias->is_contiguous(), "bias must be contiguous [N]");
    REVPP_CHECK((reinterpret_cast<uintptr_t>(bias->data_ptr()) & 15) == 0, "bias must be 16-byte aligned");
    args.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  args.aux = nullptr;
  args.aux_out = nullptr;
  args.ld_aux = 0;
  if (epi == kEpiDGelu) {
    REVPP_CHECK(aux.has_value() && aux->defined(), "DGelu epilogue needs aux (pre-activation)");
    check_cuda_bf16(*aux, "aux");
    REVPP_CHECK(aux->stride(1) == 1 && aux->size(0) >= M && aux->size(1) >= N);
    args.aux = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr());
    args.ld_aux = aux->stride(0);
  }
  if (epi == kEpiGelu && aux_out.has_value() && aux_out->defined()) {
    check_cuda_bf16(*aux_out, "aux_out");
    REVPP_CHECK(aux_out->stride(1) == 1 && aux_out->size(0) >= M && aux_out->size(1) >= N);
    args.aux_out = reinterpret_cast<__nv_bfloat16*>(aux_out->data_ptr());
    args.ld_aux = aux_out->stride(0);
  }
  args.resid = nullptr;
  args.ld_resid = 0;
  if (epi == kEpiResid) {
    REVPP_CHECK(resid.has_value() && resid->defined(), "Resid epilogue needs resid");
    check_cuda_f32(*resid, "resid");
    REVPP_CHECK(resid->stride(1) == 1 && resid->size(0) >= M && resid->size(1) >= N);
    args.resid = resid->data_ptr<float>();
    args.ld_resid = resid->stride(0);
  }
  args.sign = static_cast<float>(sign);
  args.colsum_part = nullptr;
  torch::Tensor part;
  if (colsum.has_value() && colsum->defined()) {
    REVPP_CHECK(epi == kEpiDGelu, "the fused column sum is implemented for the GELU-backward epilogue only");
    check_cuda_f32(*colsum, "colsum");
    REVPP_CHECK(colsum->is_contiguous() && colsum->numel() >= N, "colsum must hold N floats");
    // one row of partial column sums per 32 output rows, every row written by the epilogue
    part = torch::empty({(M + 31) / 32, N}, colsum->options());
    args.colsum_part = part.data_ptr<float>();
  }
  // REVPP_GEMM_RASTER=m numbers tiles m-fastest (the older order), for measurements
  static const int raster_m = [] {
    const char* e = std::getenv("REVPP_GEMM_RASTER");
    return (e != nullptr && e[0] == 'm') ? 1 : 0;
  }();
  args.raster_m = raster_m;
  args.status = status_device_ptr();

  const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap ta, tb;
  if (!a_mn) ta = make_tmap_2d(A.data_ptr(), bf, 2, K, M, A.stride(0) * 2, 64, kGemmBM, sw);
  else ta = make_tmap_2d(A.data_ptr(), bf, 2, M, K, A.stride(0) * 2, 64, kGemmBK, sw);
  if (!b_mn) tb = make_tmap_2d(B.data_ptr(), bf, 2, K, N, B.stride(0) * 2, 64, two_sm ? 128 : 256, sw);
  else tb = make_tmap_2d(B.data_ptr(), bf, 2, N, K, B.stride(0) * 2, 64, kGemmBK, sw);

  const int num_tiles = args.tiles_m * args.tiles_n * args.splits;
  cudaStream_t st = cur_stream();
  if (two_sm) {
    const int clusters = std::max(1, std::min(num_tiles, gemm_grid_sms() / 2));
    dispatch_gemm2(a_mn, b_mn, static_cast<int>(epi), ta, tb, args, 2 * clusters, st);
  } else {
    const int grid = std::min(num_tiles, gemm_grid_sms());
    dispatch_gemm(a_mn, b_mn, static_cast<int>(epi), ta, tb, args, grid, st);
  }
  if (args.colsum_part != nullptr) {
    const int rows = static_cast<int>((M + 31) / 32);
    dim3 grid(static_cast<unsigned>((N + 127) / 128), static_cast<unsigned>(std::min(8, rows)));
    gemm_colsum_reduce_kernel<<<grid, 256, 0, st>>>(args.colsum_part, colsum->data_ptr<float>(), rows,
                                                    static_cast<int>(N));
    REVPP_CHECK_LAUNCH();
  }
}

// Split count for the weight-gradient GEMM (K = tokens, long).  The persistent grid runs
// 256 x 256 tiles on SM pairs; with `pt` output tiles and s splits every pair runs
// ceil(pt s / pairs) tiles of ceil(kb / s) k-blocks, plus a fixed cost per tile (pipeline
// fill and the fp32 atomic epilogue, fitted as 16 k-blocks to a sweep of the four weight
// shapes of a BERT-Large layer at 8192 and 32768 tokens).  The split count minimising that
// makespan is taken (the smallest on ties), keeping >= 8 k-blocks per split.  At
// N x K = 3072 x 1024 over 32768 tokens this gives 3 splits: 161 us against 223 us with 1
// (48 tiles on 74 pairs).  `sms` <= 0: this device's SM count.
int64_t gemm_suggest_splits(int64_t M, int64_t N, int64_t K, int64_t sms) {
  const int64_t pt = ((M + 2 * kGemmBM - 1) / (2 * kGemmBM)) * ((N + 255) / 256);
  const int64_t kb = (K + kGemmBK - 1) / kGemmBK;
  const int64_t pairs = std::max<int64_t>(1, (sms > 0 ? sms : num_sms()) / 2);
  constexpr int64_t kTileCost = 16;
  int64_t best = 1, best_cost = -1;
  for (int64_t s = 1; s <= 16; ++s) {
    if (s > 1 && kb / s < 8) break;
    const int64_t rounds = (pt * s + pairs - 1) / pairs;
    const int64_t cost = rounds * ((kb + s - 1) / s + kTileCost);
    if (best_cost < 0 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

}  // namespace revpp
