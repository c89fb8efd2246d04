// tcgen05 / TMEM grouped GEMM for sm_100a, fed by TMA.
//
// Orientation: the weight rows are the MMA M side (128 output features per
// CTA tile) and the permuted token rows are the N side (BN = 16..256).  Decode
// batches put only a handful of tokens on each expert, and the M=128 x N=16
// instruction keeps the tensor core busy on weights streamed from HBM, while
// prefill batches use N = 256.  Accumulators live in TMEM; the epilogue reads
// them with tcgen05.ld (one TMEM lane quarter per epilogue warp).
//
// Warp roles (192 threads):
//   warps 0-3  dequantise fp8 / int4 weight tiles to bf16 in shared memory
//              during the main loop, then run the epilogue;
//   warp 4     TMA producer (one elected lane);
//   warp 5     TMEM allocator and MMA issuer (one elected lane).
// Every mbarrier wait is bounded (sb_common.cuh): a wait that runs out records
// a bit in the caller's status word and the CTA winds down instead of hanging.
//
// No load in this file uses cluster multicast: every CTA fetches its own tiles,
// so the kernel is safe on expert-parallel runs where operands may live in
// buffers filled by other GPUs.
#include <cstdlib>
#include <unordered_map>
#include <mutex>
#include <tuple>

#include "sb_gemm_common.cuh"
#include "sb_internal.h"

namespace sb {

constexpr int kTcBM = 128;
constexpr int kTcBK = 64;
constexpr int kTcThreads = 192;
// Shared memory for the pipeline stages: small column tiles (decode) keep two
// CTAs per SM (two independent TMA/MMA latency chains), large ones take one.
// Shared-memory budgets of the one-tile kernel (they set the stage count and
// so the CTAs per SM), measured on B200: the fixed-group schedule streams a
// whole expert per CTA and is fastest with 4 stages and 2 CTAs per SM (bf16
// decode, cfg2); one-tile slots (<= 64 columns) and fp8 / int4 tiles, whose
// dequant runs in the CTA's own epilogue warps, are fastest with 2 stages and
// 3-4 CTAs per SM (cfg5: +20% on the edge-value and expert GEMMs).
constexpr int kTcSmemBudgetFixed = 110 * 1024;
constexpr int kTcSmemBudgetSmallN = 50 * 1024;
constexpr int kTcSmemBudgetSmallNConvert = 64 * 1024;
constexpr int kTcSmemBudgetLargeN = 200 * 1024;

template <int BN, int WFMT, int EPI, bool kFixed>
struct TcCfg {
  static constexpr bool kGate = EPI == SB_EPI_SWIGLU;
  // interleaved SwiGLU: warps 0-1 (gate rows) hand silu(gate) to warps 2-3
  // (up rows of the same features) through a 2 KB buffer per warp pair
  static constexpr bool kIL = EPI == SB_EPI_SWIGLU_IL;
  static constexpr int kXBytes = kIL ? 2 * 2048 : 0;
  static constexpr bool kConvert = WFMT != SB_W_BF16;
  static constexpr int kABytes = kTcBM * kTcBK * 2;                       // bf16 tile
  static constexpr int kBBytes = BN * kTcBK * 2;
  static constexpr int kRawBytes = WFMT == SB_W_FP8 ? kTcBM * kTcBK : (WFMT == SB_W_INT4 ? kTcBM * kTcBK / 2 : 0);
  static constexpr int kStageBytes = kABytes * (kGate ? 2 : 1) + kBBytes + kRawBytes * (kGate ? 2 : 1);
  static constexpr int kBudget =
      BN > 64 ? kTcSmemBudgetLargeN
              : (kConvert ? kTcSmemBudgetSmallNConvert : (kFixed ? kTcSmemBudgetFixed : kTcSmemBudgetSmallN));
  static constexpr int kStagesRaw = kBudget / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : (kStagesRaw < 2 ? 2 : kStagesRaw);
  static constexpr int kTmemCols = (BN * (kGate ? 2 : 1)) <= 32 ? 32 : BN * (kGate ? 2 : 1);
  // shared memory layout (offsets from a 1024-aligned base)
  static constexpr int kOffA = 0;
  static constexpr int kOffG = kOffA + kStages * kABytes;
  static constexpr int kOffB = kOffG + (kGate ? kStages * kABytes : 0);
  static constexpr int kOffRaw = kOffB + kStages * kBBytes;
  static constexpr int kOffRawG = kOffRaw + kStages * kRawBytes;
  static constexpr int kOffBar = kOffRawG + (kGate ? kStages * kRawBytes : 0);
  static constexpr int kOffMisc = kOffBar + (3 * kStages + 2) * 8;
  // int4: the CTA's group scales (128 rows x up to 32 groups of its K range)
  static constexpr int kScaleBytes = WFMT == SB_W_INT4 ? 8192 : 0;
  static constexpr int kOffScale = kOffMisc + 64;
  static constexpr int kOffX = kOffScale + kScaleBytes;
  static constexpr int kSmemBytes = kOffX + kXBytes + 1024;  // + alignment slack
  static_assert(kTmemCols <= 512, "TMEM holds 512 columns");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "M=128 MMA needs N in [16, 256], N % 16 == 0");
};

// Two int4 weights -- the low nibbles of byte p of w (element 2p) and of byte
// p of w >> 4 (element 2p + 1) -- as the bf16x2 bit patterns of 128 + (n ^ 8),
// n the raw nibble: exponent 2^7 with u = n ^ 8 = q + 8 in the low mantissa
// bits, exact.  One byte permute and one three-input logic op per pair.
template <int kP>
SB_DEVINL uint32_t int4x2_biased_bf16x2(uint32_t w, uint32_t w_shr4) {
  constexpr uint32_t kSel = kP | (kP << 4) | ((4 + kP) << 8) | ((4 + kP) << 12);
  return (__byte_perm(w, w_shr4, kSel) & 0x000F000Fu) ^ 0x43084308u;
}

// One 16-byte chunk of a raw fp8 tile row (16 weights, e4m3) -> two 16-byte
// bf16 chunks of the swizzled tile: row `row`, 16-byte chunk c16 of its 64 bytes.
SB_DEVINL void convert_fp8_chunk(const uint4 v, uint8_t* dst, int row, int c16) {
  const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
  uint32_t out[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(b[2 * j] | (b[2 * j + 1] << 8)), __NV_E4M3);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    const __nv_bfloat162 bb = __floats2bfloat162_rn(f.x, f.y);
    out[j] = *reinterpret_cast<const uint32_t*>(&bb);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int kc = c16 * 2 + h;  // 16-byte chunk (8 bf16) index along k
    *reinterpret_cast<uint4*>(dst + row * 128 + ((kc ^ (row & 7)) << 4)) =
        make_uint4(out[4 * h], out[4 * h + 1], out[4 * h + 2], out[4 * h + 3]);
  }
}

// One 16-byte chunk of a raw int4 tile row (32 weights) with its group scale
// -> four 16-byte bf16 chunks of the swizzled tile (row `row`, chunk c16 of
// its 32 bytes).  Each weight is bf16(q * s) with one rounding, as the
// CUDA-core engine and the oracle compute it: (128 + u) - 136 is exact in
// bf16 and the bf16x2 multiply rounds the exact product once.
SB_DEVINL void convert_int4_chunk(const uint4 v, const __nv_bfloat16 sb, uint8_t* dst, int row, int c16) {
  const __nv_bfloat162 bias = __float2bfloat162_rn(136.f);
  const __nv_bfloat162 s2 = __bfloat162bfloat162(sb);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t h = w[i] >> 4;
    uint32_t pr[4] = {int4x2_biased_bf16x2<0>(w[i], h), int4x2_biased_bf16x2<1>(w[i], h),
                      int4x2_biased_bf16x2<2>(w[i], h), int4x2_biased_bf16x2<3>(w[i], h)};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 qv = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&pr[j]), bias);
      const __nv_bfloat162 r = __hmul2(qv, s2);
      out[4 * i + j] = *reinterpret_cast<const uint32_t*>(&r);
    }
  }
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const int kc = c16 * 4 + h;
    *reinterpret_cast<uint4*>(dst + row * 128 + ((kc ^ (row & 7)) << 4)) =
        make_uint4(out[4 * h], out[4 * h + 1], out[4 * h + 2], out[4 * h + 3]);
  }
}

// Convert the raw fp8 / int4 tile of this stage into the swizzled bf16 tile.
// int4: the group scale of (row, k0) comes from `s_scale[row * s_ngr + k0 /
// group_size - s_g0]` in shared memory when s_scale is given, else from global
// memory.
template <int WFMT>
SB_DEVINL void convert_tile(const uint8_t* raw, uint8_t* dst, const sb_grouped_gemm_args& p,
                            const void* scales, int64_t arow0, int k0, int tid,
                            const __nv_bfloat16* s_scale = nullptr, int s_ngr = 0, int s_g0 = 0) {
  if (WFMT == SB_W_FP8) {
    // 128 rows x 64 bytes; item = (row, 16-byte chunk): 512 items over 128 threads.
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int item = tid + 128 * q;
      const int row = item >> 2, c16 = item & 3;
      convert_fp8_chunk(*reinterpret_cast<const uint4*>(raw + row * 64 + c16 * 16), dst, row, c16);
    }
  } else {
    // 128 rows x 32 bytes; item = (row, 16-byte chunk): 256 items over 128 threads.
    const int groups = static_cast<int>(p.lda / p.group_size);
    const int gk = k0 / p.group_size;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int item = tid + 128 * q;
      const int row = item >> 1, c16 = item & 1;
      const int64_t arow = arow0 + row;
      __nv_bfloat16 sb;
      if (s_scale)
        sb = s_scale[row * s_ngr + gk - s_g0];
      else
        sb = arow < p.a_rows_total ? static_cast<const __nv_bfloat16*>(scales)[arow * groups + gk]
                                   : __float2bfloat16_rn(0.f);
      convert_int4_chunk(*reinterpret_cast<const uint4*>(raw + row * 32 + c16 * 16), sb, dst, row, c16);
    }
  }
}

// Modes.  kFixed (decode-size column tiles): CTA (m-tile, group) covers every
// row tile of its group, and its first weight tiles are requested before the
// dependency wait -- the weights do not depend on the preceding kernel, so
// they stream in while that kernel finishes.  kGather: the token rows are
// fetched with tile::gather4 straight from the unpermuted activation matrix
// (no permuted copy in HBM): each gather writes four whole 128-byte rows
// (512 bytes, 512-byte aligned) into the same 128-byte swizzled layout a tiled
// load produces.  Otherwise (large tiles) a CTA takes one (group, row tile)
// slot of the upper-bound grid and B is one tiled TMA load.
template <int BN, int WFMT, int EPI, bool kFixed, bool kGather>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmG,
               const __grid_constant__ CUtensorMap tmB, const sb_grouped_gemm_args p) {
  using C = TcCfg<BN, WFMT, EPI, kFixed>;
  constexpr int S = C::kStages;
  static_assert(!kGather || BN <= 64, "gathers are issued by the lanes of one warp (BN/4 <= 32)");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + S;
  uint64_t* conv = empty + S;
  uint64_t* acc_full = conv + S;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  int* s_sched = reinterpret_cast<int*>(smem + C::kOffMisc + 16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * kTcBM;
  const int ks = p.k / p.splits;
  const int kb = blockIdx.z * ks;
  const int nk = ks / kTcBK;

  // ---- set-up that reads no predecessor output (runs before the dependency wait)
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 128);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 128);
    fence_barrier_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (C::kGate) tma_prefetch_desc(&tmG);
  }
  __syncthreads();
  int pre = 0;  // weight tiles requested before the wait (kFixed)
  constexpr uint32_t kTxA = (C::kConvert ? C::kRawBytes : C::kABytes) * (C::kGate ? 2 : 1);
  if (kFixed && warp == 4 && lane == 0) {
    const int64_t arow = static_cast<int64_t>(blockIdx.y) * p.a_group_rows + m0;
    pre = nk < S ? nk : S;
    for (int it = 0; it < pre; ++it) {
      mbar_add_tx(&full[it], kTxA);  // the stage's arrival (with its B bytes) comes after the wait
      const int k0 = kb + it * kTcBK;
      const int acol = WFMT == SB_W_INT4 ? k0 / 2 : k0;
      uint8_t* adst = C::kConvert ? smem + C::kOffRaw + it * C::kRawBytes : smem + C::kOffA + it * C::kABytes;
      tma_load_2d(adst, &tmA, &full[it], acol, static_cast<int>(arow));
      if (C::kGate) {
        uint8_t* gdst = C::kConvert ? smem + C::kOffRawG + it * C::kRawBytes : smem + C::kOffG + it * C::kABytes;
        tma_load_2d(gdst, &tmG, &full[it], acol, static_cast<int>(arow));
      }
    }
  }
  // int4, fixed schedule: this CTA's group scales into shared memory, also
  // before the wait (weights and scales do not depend on the previous kernel)
  __nv_bfloat16* s_scale = nullptr;
  int s_ngr = 0, s_g0 = 0;
  if (kFixed && WFMT == SB_W_INT4) {
    const int gs = p.group_size;
    s_g0 = kb / gs;
    s_ngr = (kb + ks + gs - 1) / gs - s_g0;
    if (s_ngr * kTcBM * 2 <= C::kScaleBytes) {
      s_scale = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffScale);
      if (warp < 4) {
        const int groups = static_cast<int>(p.lda / gs);
        const int64_t arow0s = static_cast<int64_t>(blockIdx.y) * p.a_group_rows + m0;
        const __nv_bfloat16* sc = static_cast<const __nv_bfloat16*>(p.a_scale);
        for (int i = tid; i < s_ngr * kTcBM; i += 128) {
          const int row = i / s_ngr, gi = i - row * s_ngr;
          const int64_t arow = arow0s + row;
          s_scale[i] = arow < p.a_rows_total ? sc[arow * groups + s_g0 + gi] : __float2bfloat16_rn(0.f);
        }
      }
    }
  }
  pdl_wait();
  pdl_trigger();

  // ---- schedule
  if (kFixed) {
    if (tid == 0) {
      const int g = blockIdx.y;
      s_sched[0] = g;
      s_sched[1] = group_offset(p.offsets, g, p.max_rows);
      s_sched[2] = min(group_offset(p.offsets, g + 1, p.max_rows), p.max_rows);
    }
  } else if (warp == 0) {
    int g, n0, n_end;
    const bool ok = schedule_tile(p.offsets, p.num_groups, BN, blockIdx.y, g, n0, n_end, p.max_rows);
    if (lane == 0) {
      s_sched[0] = ok ? g : -1;
      s_sched[1] = n0;
      s_sched[2] = min(min(n_end, p.max_rows), n0 + BN);
    }
  }
  __syncthreads();
  const int g = s_sched[0];
  const int n0 = s_sched[1], n_end = s_sched[2];
  if (!kFixed && g < 0) return;  // surplus slot of the upper-bound grid
  const int rows = n_end - n0;
  if (kFixed && rows <= 0) {
    // A group without rows: arrive on the stages whose weights were requested
    // and let those copies land before exiting.
    if (warp == 4 && lane == 0) {
      for (int it = 0; it < pre; ++it) mbar_arrive(&full[it]);
      for (int it = 0; it < pre; ++it)
        if (!mbar_wait(&full[it], 0, p.status, SB_DEVERR_DRAIN)) break;
    }
    return;
  }
  const int ntile = kFixed ? (rows + BN - 1) / BN : 1;
  const int total_it = ntile * nk;
  const int64_t arow0 = static_cast<int64_t>(g) * p.a_group_rows + m0;

  if (warp == 5) {
    tmem_alloc(s_tmem, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 4) {
    // ---------------------------------------------------------------- producer
    int issued = 0;
    int rix[4] = {0, 0, 0, 0};  // kGather: the four token rows this lane gathers (lanes < BN/4)
    for (int it = 0; it < total_it; ++it) {
      const int t = it / nk, kk = it - t * nk;
      const int s = it % S;
      const uint32_t ph = (it / S) & 1;
      const int k0 = kb + kk * kTcBK;
      const int nrow = n0 + t * BN;
      // Only the tile's valid rows are fetched: 4-row gathers, or 16-row tiled
      // boxes on the fixed-group schedule; the rest of the tile is never read.
      const int tval = min(BN, n_end - nrow);
      const int nb = kGather ? (tval + 3) / 4 : (kFixed ? (tval + 15) / 16 : 1);
      const uint32_t tx_b = kGather ? nb * 512u : (kFixed ? nb * 2048u : static_cast<uint32_t>(C::kBBytes));
      if (kGather && kk == 0 && lane < nb) {
        // token rows of this tile; rows past the group's end repeat its last row (discarded)
#pragma unroll
        for (int r = 0; r < 4; ++r) rix[r] = p.x_row_index[min(nrow + 4 * lane + r, n_end - 1)];
      }
      bool ok = true;
      if (lane == 0) {
        if (kFixed && it < pre) {
          mbar_expect_tx(&full[s], tx_b);  // weights already requested before the wait
        } else {
          ok = mbar_wait(&empty[s], ph ^ 1, p.status, SB_DEVERR_MMA_WAIT);
          if (ok) {
            mbar_expect_tx(&full[s], kTxA + tx_b);
            const int acol = WFMT == SB_W_INT4 ? k0 / 2 : k0;
            uint8_t* adst = C::kConvert ? smem + C::kOffRaw + s * C::kRawBytes : smem + C::kOffA + s * C::kABytes;
            tma_load_2d(adst, &tmA, &full[s], acol, static_cast<int>(arow0));
            if (C::kGate) {
              uint8_t* gdst = C::kConvert ? smem + C::kOffRawG + s * C::kRawBytes : smem + C::kOffG + s * C::kABytes;
              tma_load_2d(gdst, &tmG, &full[s], acol, static_cast<int>(arow0));
            }
          }
        }
        if (ok && !kGather) {
          if (kFixed)
            for (int j = 0; j < nb; ++j)
              tma_load_2d(smem + C::kOffB + s * C::kBBytes + j * 2048, &tmB, &full[s], k0, nrow + 16 * j);
          else
            tma_load_2d(smem + C::kOffB + s * C::kBBytes, &tmB, &full[s], k0, nrow);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (kGather) {
        __syncwarp();
        if (lane < nb)
          tma_gather4(smem + C::kOffB + s * C::kBBytes + lane * 512, &tmB, &full[s], k0, rix[0], rix[1], rix[2], rix[3]);
      }
      ++issued;
    }
    // Drain: every issued copy must have landed before the CTA may exit.
    if (lane == 0)
      for (int it = issued - S > 0 ? issued - S : 0; it < issued; ++it)
        if (!mbar_wait(&full[it % S], (it / S) & 1, p.status, SB_DEVERR_DRAIN)) break;
    __syncwarp();
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kTcBM, BN);
      bool ok = true;
      for (int t = 0; t < ntile && ok; ++t) {
        if (t > 0) ok = mbar_wait(acc_empty, (t - 1) & 1, p.status, SB_DEVERR_EPI_WAIT);
        tc_fence_after();
        for (int kk = 0; kk < nk && ok; ++kk) {
          const int it = t * nk + kk;
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          ok = C::kConvert ? mbar_wait(&conv[s], ph, p.status, SB_DEVERR_CONV_WAIT)
                           : mbar_wait(&full[s], ph, p.status, SB_DEVERR_TMA_WAIT);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + C::kOffA + s * C::kABytes);
          const uint32_t g_base = smem_u32(smem + C::kOffG + s * C::kABytes);
          const uint32_t b_base = smem_u32(smem + C::kOffB + s * C::kBBytes);
#pragma unroll
          for (int j = 0; j < kTcBK / 16; ++j) {
            const uint64_t bdesc = smem_desc_k_sw128(b_base + j * 32);
            const uint32_t accum = (kk > 0 || j > 0) ? 1u : 0u;
            tc_mma_bf16(tmem, smem_desc_k_sw128(a_base + j * 32), bdesc, idesc, accum);
            if (C::kGate) tc_mma_bf16(tmem + BN, smem_desc_k_sw128(g_base + j * 32), bdesc, idesc, accum);
          }
          tc_commit(&empty[s]);
        }
        tc_commit(acc_full);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- dequant + epilogue
    const int mloc = warp * 32 + lane;
    const int m = m0 + mloc;
    const int64_t arow = arow0 + mloc;
    const bool mvalid = m < p.m_rows && arow < p.a_rows_total;
    const float sa = ((WFMT == SB_W_FP8 || (WFMT == SB_W_BF16 && p.a_scale)) && mvalid) ? static_cast<const float*>(p.a_scale)[arow] : 1.f;
    const float sg = (C::kGate && (WFMT == SB_W_FP8 || (WFMT == SB_W_BF16 && p.a_gate_scale)) && mvalid) ? static_cast<const float*>(p.a_gate_scale)[arow] : 1.f;
    const float bias = (p.bias && mvalid && blockIdx.z == 0) ? p.bias[static_cast<int64_t>(g) * p.bias_group_stride + m] : 0.f;
    const float bgate = (C::kGate && p.bias_gate && mvalid) ? p.bias_gate[static_cast<int64_t>(g) * p.bias_group_stride + m] : 0.f;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    bool live = true;
    for (int t = 0; t < ntile && live; ++t) {
      if (C::kConvert) {
        for (int kk = 0; kk < nk; ++kk) {
          const int it = t * nk + kk;
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          if (!mbar_wait(&full[s], ph, p.status, SB_DEVERR_TMA_WAIT)) { live = false; break; }
          const int k0 = kb + kk * kTcBK;
          convert_tile<WFMT>(smem + C::kOffRaw + s * C::kRawBytes, smem + C::kOffA + s * C::kABytes, p,
                             p.a_scale, arow0, k0, tid, s_scale, s_ngr, s_g0);
          if (C::kGate)
            convert_tile<WFMT>(smem + C::kOffRawG + s * C::kRawBytes, smem + C::kOffG + s * C::kABytes, p,
                               p.a_gate_scale, arow0, k0, tid);
          fence_proxy_async_smem();
          mbar_arrive(&conv[s]);
        }
      }
      const int tn0 = n0 + t * BN;
      const int tend = min(tn0 + BN, n_end);
      // LINEAR row scales of the tile, one per lane and 32 columns, read before
      // the accumulator wait so their latency overlaps the MMAs
      float rsv[BN >= 32 ? BN / 32 : 1];
#pragma unroll
      for (int i = 0; i < (BN >= 32 ? BN / 32 : 1); ++i) {
        const int r = tn0 + i * 32 + lane;
        rsv[i] = (EPI == SB_EPI_LINEAR && p.row_scale && r < tend && i * 32 + lane < BN) ? p.row_scale[r] : 1.f;
      }
      // tcgen05.ld is warp-collective: every lane must take the same branch.
      live = __all_sync(0xffffffffu, live && mbar_wait(acc_full, t & 1, p.status, SB_DEVERR_EPI_WAIT));
      // interleaved SwiGLU: both warps of a (gate, up) pair take the same path
      if (C::kIL) live = named_bar_and(1 + (warp & 1), 64, live);
      tc_fence_after();
      if (!live) break;
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 16) {
        if (tn0 + c0 >= tend) break;  // warp-uniform
        float v[16], vg[16], o[16];
        tmem_ld16(lane_addr + c0, v);
        if (C::kGate) tmem_ld16(lane_addr + BN + c0, vg);
        if constexpr (C::kIL) {
          // warps 0-1 hold the gate rows of the tile's 64 features, warps 2-3
          // their up rows: silu(gate) goes across through shared memory
          float* xb = reinterpret_cast<float*>(smem + C::kOffX) + (warp & 1) * 512;
          if (warp < 2) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xb[j * 32 + lane] = silu_bf16out(v[j] * sa + bias);
            named_bar_sync(1 + (warp & 1), 64);  // values ready
            named_bar_sync(1 + (warp & 1), 64);  // values taken
            continue;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = v[j] * sa + bias;
          named_bar_sync(1 + (warp & 1), 64);
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] *= xb[j * 32 + lane];
          named_bar_sync(1 + (warp & 1), 64);
          if (!mvalid) continue;
          const int nvalid = tend - (tn0 + c0);
          const int64_t base = static_cast<int64_t>(tn0 + c0) * p.ldo + m0 / 2 + (warp - 2) * 32 + lane;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (nvalid < 16 && j >= nvalid) break;
            static_cast<__nv_bfloat16*>(p.out)[base + static_cast<int64_t>(j) * p.ldo] = __float2bfloat16_rn(o[j]);
          }
          continue;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float x = v[j] * sa + bias;
          if (EPI == SB_EPI_LINEAR)
            o[j] = x * __shfl_sync(0xffffffffu, rsv[(c0 + j) >> 5], (c0 + j) & 31);
          else if (EPI == SB_EPI_GELU)
            o[j] = gelu_bf16out(x);
          else
            o[j] = silu_bf16out(vg[j] * sg + bgate) * x;
        }
        if (!mvalid) continue;
        const int nvalid = tend - (tn0 + c0);
        const int64_t base = static_cast<int64_t>(tn0 + c0) * p.ldo + m;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (nvalid < 16 && j >= nvalid) break;
          if (EPI == SB_EPI_LINEAR)
            static_cast<float*>(p.out)[blockIdx.z * p.split_stride + base + static_cast<int64_t>(j) * p.ldo] = o[j];
          else
            static_cast<__nv_bfloat16*>(p.out)[base + static_cast<int64_t>(j) * p.ldo] = __float2bfloat16_rn(o[j]);
        }
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ persistent large-tile GEMM
//
// Prefill-size problems (many row tiles per group): one CTA per SM walks the
// tile list (group, row tile, 128-feature tile; feature tile fastest so a token
// tile is reused from L2 by all feature tiles), with the TMA pipeline running
// continuously across tiles and two TMEM accumulators, so the epilogue of tile
// i overlaps the MMAs of tile i+1.  Eight epilogue warps, two per TMEM lane
// quarter (one per half of the tile's columns), keep the epilogue shorter than
// a tile's MMAs; fp8 / int4 tiles are dequantised by four dedicated warps.
// Warps: 0-3 and 6-9 epilogue, 4 TMA, 5 MMA (+TMEM), 10-13 dequant.
template <int BN, int WFMT, int EPI>
struct PCfg {
  static constexpr bool kGate = EPI == SB_EPI_SWIGLU;
  static constexpr bool kIL = EPI == SB_EPI_SWIGLU_IL;  // four gate/up warp pairs, 2 KB each
  static constexpr int kXBytes = kIL ? 4 * 2048 : 0;
  static constexpr bool kConvert = WFMT != SB_W_BF16;
  static constexpr int kABytes = kTcBM * kTcBK * 2;
  static constexpr int kBBytes = BN * kTcBK * 2;
  static constexpr int kRawBytes = WFMT == SB_W_FP8 ? kTcBM * kTcBK : (WFMT == SB_W_INT4 ? kTcBM * kTcBK / 2 : 0);
  static constexpr int kStageBytes = kABytes * (kGate ? 2 : 1) + kBBytes + kRawBytes * (kGate ? 2 : 1);
  static constexpr int kStagesRaw = (212 * 1024 - kXBytes) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 6 ? 6 : (kStagesRaw < 2 ? 2 : kStagesRaw);
  static constexpr int kAccCols = BN * (kGate ? 2 : 1);
  static constexpr int kTmemCols = 2 * kAccCols;
  static constexpr int kEpiThreads = 256;
  static constexpr int kThreads = kConvert ? 448 : 320;
  static constexpr int kOffA = 0;
  static constexpr int kOffG = kOffA + kStages * kABytes;
  static constexpr int kOffB = kOffG + (kGate ? kStages * kABytes : 0);
  static constexpr int kOffRaw = kOffB + kStages * kBBytes;
  static constexpr int kOffRawG = kOffRaw + kStages * kRawBytes;
  static constexpr int kOffBar = kOffRawG + (kGate ? kStages * kRawBytes : 0);
  static constexpr int kOffMisc = kOffBar + (3 * kStages + 4) * 8;
  static constexpr int kOffPrefix = kOffMisc + 64;                  // int[kMaxG + 1]
  static constexpr int kMaxG = 256;
  static constexpr int kOffOffsets = kOffPrefix + (kMaxG + 1) * 4;  // int[kMaxG + 1]: group row offsets
  static constexpr int kOffX = kOffOffsets + (kMaxG + 1) * 4;
  static constexpr int kSmemBytes = kOffX + kXBytes + 1024;
  static_assert(kTmemCols <= 512, "two accumulators must fit the 512 TMEM columns");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
};

// MMA width for a tile holding `rows` valid token rows (the last tile of a
// group is usually partial): rows rounded up to 16, at most BN -- the tensor
// core then spends no cycles on the empty columns of short tiles.
template <int BN>
SB_DEVINL int tile_mma_n(int rows) {
  const int n = (rows + 15) & ~15;
  return n < 16 ? 16 : (n > BN ? BN : n);
}

// Tile t -> (group, row tile, feature tile) from the per-group tile prefix.
SB_DEVINL void decode_tile(const int* prefix, int G, int m_tiles, int t, int& g, int& nt, int& mt) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {  // largest g with prefix[g] <= t
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= t) lo = mid; else hi = mid - 1;
  }
  g = lo;
  const int local = t - prefix[g];
  nt = local / m_tiles;
  mt = local - nt * m_tiles;
}

template <int BN, int WFMT, int EPI>
__global__ void __launch_bounds__(PCfg<BN, WFMT, EPI>::kThreads, 1)
tc_gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmG,
                          const __grid_constant__ CUtensorMap tmB, const sb_grouped_gemm_args p) {
  using C = PCfg<BN, WFMT, EPI>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + S;
  uint64_t* conv = empty + S;
  uint64_t* acc_full = conv + S;     // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  int* s_total = reinterpret_cast<int*>(smem + C::kOffMisc + 16);
  int* prefix = reinterpret_cast<int*>(smem + C::kOffPrefix);
  int* s_off = reinterpret_cast<int*>(smem + C::kOffOffsets);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.num_groups;
  const int m_tiles = (p.m_rows + kTcBM - 1) / kTcBM;
  const int nk = p.k / kTcBK;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 128);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], C::kEpiThreads);
    }
    fence_barrier_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (C::kGate) tma_prefetch_desc(&tmG);
  }
  pdl_wait();
  pdl_trigger();
  if (warp == 0) {
    // per-group tile counts -> exclusive prefix (warp scan, 32 groups at a time)
    int seen = 0;
    for (int base = 0; base < G; base += 32) {
      const int gi = base + lane;
      int tiles = 0;
      if (gi < G) {
        const int o0 = group_offset(p.offsets, gi, p.max_rows), o1 = group_offset(p.offsets, gi + 1, p.max_rows);
        s_off[gi] = o0;
        if (gi == G - 1) s_off[G] = o1;
        const int lo = min(o0, p.max_rows), hi = min(o1, p.max_rows);
        tiles = hi > lo ? (hi - lo + BN - 1) / BN * m_tiles : 0;
      }
      int incl = tiles;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += t;
      }
      if (gi < G) prefix[gi] = seen + incl - tiles;
      seen += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      prefix[G] = seen;
      *s_total = seen;
    }
  }
  __syncthreads();
  const int total = *s_total;
  if (static_cast<int>(blockIdx.x) >= total) return;  // no tile for this CTA
  const int my_tiles = (total - static_cast<int>(blockIdx.x) + gridDim.x - 1) / gridDim.x;

  if (warp == 5) {
    tmem_alloc(s_tmem, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 4) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      constexpr uint32_t kTx = (C::kConvert ? C::kRawBytes : C::kABytes) * (C::kGate ? 2 : 1) + C::kBBytes;
      int it = 0;
      bool ok = true;
      for (int j = 0; j < my_tiles && ok; ++j) {
        int g, nt, mt;
        decode_tile(prefix, G, m_tiles, blockIdx.x + j * gridDim.x, g, nt, mt);
        const int64_t arow = static_cast<int64_t>(g) * p.a_group_rows + mt * kTcBM;
        const int nrow = s_off[g] + nt * BN;
        for (int kk = 0; kk < nk; ++kk, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, p.status, SB_DEVERR_MMA_WAIT)) { ok = false; break; }
          mbar_expect_tx(&full[s], kTx);
          const int k0 = kk * kTcBK;
          const int acol = WFMT == SB_W_INT4 ? k0 / 2 : k0;
          uint8_t* adst = C::kConvert ? smem + C::kOffRaw + s * C::kRawBytes : smem + C::kOffA + s * C::kABytes;
          tma_load_2d(adst, &tmA, &full[s], acol, static_cast<int>(arow));
          if (C::kGate) {
            uint8_t* gdst = C::kConvert ? smem + C::kOffRawG + s * C::kRawBytes : smem + C::kOffG + s * C::kABytes;
            tma_load_2d(gdst, &tmG, &full[s], acol, static_cast<int>(arow));
          }
          tma_load_2d(smem + C::kOffB + s * C::kBBytes, &tmB, &full[s], k0, nrow);
        }
      }
      for (int i = it - S > 0 ? it - S : 0; i < it; ++i)  // drain
        if (!mbar_wait(&full[i % S], (i / S) & 1, p.status, SB_DEVERR_DRAIN)) break;
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int j = 0; j < my_tiles && ok; ++j) {
        const int buf = j & 1;
        int g, nt, mt;
        decode_tile(prefix, G, m_tiles, blockIdx.x + j * gridDim.x, g, nt, mt);
        const int tile_n0 = s_off[g] + nt * BN;
        const int tile_end = min(min(s_off[g + 1], p.max_rows), tile_n0 + BN);
        const uint32_t idesc = idesc_bf16_f32(kTcBM, tile_mma_n<BN>(tile_end - tile_n0));
        if (!mbar_wait(&acc_empty[buf], ((j >> 1) & 1) ^ 1, p.status, SB_DEVERR_EPI_WAIT)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * C::kAccCols;
        for (int kk = 0; kk < nk; ++kk, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          ok = C::kConvert ? mbar_wait(&conv[s], ph, p.status, SB_DEVERR_CONV_WAIT)
                           : mbar_wait(&full[s], ph, p.status, SB_DEVERR_TMA_WAIT);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + C::kOffA + s * C::kABytes);
          const uint32_t g_base = smem_u32(smem + C::kOffG + s * C::kABytes);
          const uint32_t b_base = smem_u32(smem + C::kOffB + s * C::kBBytes);
#pragma unroll
          for (int q = 0; q < kTcBK / 16; ++q) {
            const uint64_t bdesc = smem_desc_k_sw128(b_base + q * 32);
            const uint32_t accum = (kk > 0 || q > 0) ? 1u : 0u;
            tc_mma_bf16(acc, smem_desc_k_sw128(a_base + q * 32), bdesc, idesc, accum);
            if (C::kGate) tc_mma_bf16(acc + BN, smem_desc_k_sw128(g_base + q * 32), bdesc, idesc, accum);
          }
          tc_commit(&empty[s]);
        }
        tc_commit(&acc_full[buf]);
      }
    }
    __syncwarp();
  } else if (warp >= 10) {
    // ---------------------------------------------------------------- dequant (fp8 / int4)
    if (C::kConvert) {
      const int ctid = tid - 320;
      int it = 0;
      for (int j = 0; j < my_tiles; ++j) {
        int g, nt, mt;
        decode_tile(prefix, G, m_tiles, blockIdx.x + j * gridDim.x, g, nt, mt);
        const int64_t arow0 = static_cast<int64_t>(g) * p.a_group_rows + mt * kTcBM;
        bool ok = true;
        for (int kk = 0; kk < nk; ++kk, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, p.status, SB_DEVERR_TMA_WAIT)) { ok = false; break; }
          const int k0 = kk * kTcBK;
          convert_tile<WFMT>(smem + C::kOffRaw + s * C::kRawBytes, smem + C::kOffA + s * C::kABytes, p,
                             p.a_scale, arow0, k0, ctid);
          if (C::kGate)
            convert_tile<WFMT>(smem + C::kOffRawG + s * C::kRawBytes, smem + C::kOffG + s * C::kABytes, p,
                               p.a_gate_scale, arow0, k0, ctid);
          fence_proxy_async_smem();
          mbar_arrive(&conv[s]);
        }
        if (!ok) break;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 0-3, 6-9)
    // A warp reads the TMEM lane quarter warp % 4 (output features) and one half
    // of the tile's columns (tokens).
    constexpr int HB = BN / 2;
    const int quarter = warp & 3;
    const int half = warp < 4 ? 0 : 1;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + half * HB;
    for (int j = 0; j < my_tiles; ++j) {
      int g, nt, mt;
      decode_tile(prefix, G, m_tiles, blockIdx.x + j * gridDim.x, g, nt, mt);
      const int buf = j & 1;
      // per-tile operands first: their loads overlap the wait for the accumulator
      const int m = mt * kTcBM + quarter * 32 + lane;
      const int64_t arow = static_cast<int64_t>(g) * p.a_group_rows + m;
      const bool mvalid = m < p.m_rows && arow < p.a_rows_total;
      const float sa = ((WFMT == SB_W_FP8 || (WFMT == SB_W_BF16 && p.a_scale)) && mvalid) ? static_cast<const float*>(p.a_scale)[arow] : 1.f;
      const float sg = (C::kGate && (WFMT == SB_W_FP8 || (WFMT == SB_W_BF16 && p.a_gate_scale)) && mvalid) ? static_cast<const float*>(p.a_gate_scale)[arow] : 1.f;
      const float bias = (p.bias && mvalid) ? p.bias[static_cast<int64_t>(g) * p.bias_group_stride + m] : 0.f;
      const float bgate = (C::kGate && p.bias_gate && mvalid) ? p.bias_gate[static_cast<int64_t>(g) * p.bias_group_stride + m] : 0.f;
      const int tn0 = s_off[g] + nt * BN + half * HB;
      const int tend = min(min(s_off[g] + nt * BN + BN, s_off[g + 1]), p.max_rows);
      // LINEAR: the half's row scales, one per lane and 32 columns
      float rsv[HB / 32];
#pragma unroll
      for (int i = 0; i < HB / 32; ++i) {
        const int r = tn0 + i * 32 + lane;
        rsv[i] = (EPI == SB_EPI_LINEAR && p.row_scale && r < tend) ? p.row_scale[r] : 1.f;
      }
      bool ready = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (j >> 1) & 1, p.status, SB_DEVERR_EPI_WAIT));
      // interleaved SwiGLU: quarters 0-1 hold gate rows, 2-3 the up rows of the
      // same features; warp pair (quarter q, q + 2) of each column half
      const int xpair = half * 2 + (quarter & 1);
      if (C::kIL) ready = named_bar_and(1 + xpair, 64, ready);
      tc_fence_after();
      if (!ready) break;
      const uint32_t acc_addr = lane_addr + buf * C::kAccCols;
#pragma unroll
      for (int c0 = 0; c0 < HB; c0 += 16) {
        if (tn0 + c0 >= tend) break;  // warp-uniform
        float v[16], vg[16], o[16];
        tmem_ld16(acc_addr + c0, v);
        if (C::kGate) tmem_ld16(acc_addr + BN + c0, vg);
        if constexpr (C::kIL) {
          float* xb = reinterpret_cast<float*>(smem + C::kOffX) + xpair * 512;
          if (quarter < 2) {
#pragma unroll
            for (int q = 0; q < 16; ++q) xb[q * 32 + lane] = silu_bf16out(v[q] * sa + bias);
            named_bar_sync(1 + xpair, 64);
            named_bar_sync(1 + xpair, 64);
            continue;
          }
#pragma unroll
          for (int q = 0; q < 16; ++q) o[q] = v[q] * sa + bias;
          named_bar_sync(1 + xpair, 64);
#pragma unroll
          for (int q = 0; q < 16; ++q) o[q] *= xb[q * 32 + lane];
          named_bar_sync(1 + xpair, 64);
          if (!mvalid) continue;
          const int nvalid = tend - (tn0 + c0);
          const int64_t base = static_cast<int64_t>(tn0 + c0) * p.ldo + mt * (kTcBM / 2) + (quarter - 2) * 32 + lane;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            if (nvalid < 16 && q >= nvalid) break;
            static_cast<__nv_bfloat16*>(p.out)[base + static_cast<int64_t>(q) * p.ldo] = __float2bfloat16_rn(o[q]);
          }
          continue;
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float x = v[q] * sa + bias;
          if (EPI == SB_EPI_LINEAR)
            o[q] = x * __shfl_sync(0xffffffffu, rsv[(c0 + q) >> 5], (c0 + q) & 31);
          else if (EPI == SB_EPI_GELU)
            o[q] = gelu_bf16out(x);
          else
            o[q] = silu_bf16out(vg[q] * sg + bgate) * x;
        }
        if (!mvalid) continue;
        const int nvalid = tend - (tn0 + c0);
        const int64_t base = static_cast<int64_t>(tn0 + c0) * p.ldo + m;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if (nvalid < 16 && q >= nvalid) break;
          if (EPI == SB_EPI_LINEAR)
            static_cast<float*>(p.out)[base + static_cast<int64_t>(q) * p.ldo] = o[q];
          else
            static_cast<__nv_bfloat16*>(p.out)[base + static_cast<int64_t>(q) * p.ldo] = __float2bfloat16_rn(o[q]);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ quantised decode GEMM
//
// fp8 / int4 weights with few token rows per group (decode batches; a
// Zipf-skewed router still sends up to every token to a few experts).  A
// tcgen05.mma of M=128, K=16 keeps the tensor pipe busy about as long at N=16
// as at N=256, so here the roles are swapped: the converted weights are the B
// operand (N = 256 weight rows per MMA) and the token rows the A operand
// (M = 128; rows past the item's tokens are never stored) -- twice the weights
// per MMA of a weights-as-A tile.  A persistent CTA per SM walks the
// (group, 128-token chunk, 256-weight-row tile) items, weight tile fastest.
// Packed weight tiles have a ring of their own; two groups of converter warps
// take alternate stages, so one group's conversion overlaps the other's waits.
// int4 group scales of an item (256 consecutive rows of the scale matrix, one
// contiguous block) come with one bulk copy into a double-buffered slot.  Two
// TMEM accumulators of 256 columns: the epilogue of item i overlaps the MMAs
// of item i+1; an epilogue thread holds one token row of the item.
// LINEAR outputs may be K-split (p.splits partial sums, as the other
// schedules), which multiplies the items of small problems.
// Warps: 0-3 epilogue, 4-19 convert (two groups of eight), 20 weight TMA,
// 21 MMA (+TMEM), 22 token-row TMA (16-row boxes, one 128-row box for items
// of more than 32 rows, or tile::gather4).
template <int WFMT, int EPI>
struct QCfg {
  static constexpr bool kIL = EPI == SB_EPI_SWIGLU_IL;
  static constexpr int kWRows = 256;                  // weight rows per item (MMA N)
  static constexpr int kTokM = 128;                   // token rows per item (MMA M)
  static constexpr int kWBytes = kWRows * kTcBK * 2;  // converted weights of a stage (B operand)
  static constexpr int kXBytes = kTokM * kTcBK * 2;   // token rows of a stage (A operand)
  static constexpr int kRawBytes = WFMT == SB_W_FP8 ? kWRows * kTcBK : kWRows * kTcBK / 2;
  // Ring depths.  The two converter groups take the stages of even / odd
  // global index: with an even raw ring every raw slot stays with one group,
  // so a group never polls a slot's barrier two phases ahead of it (a parity
  // wait cannot tell those apart).  The three converted stages alternate
  // between the groups, which is safe because a group reaches stage i only
  // after its stage i - 2, whose wait saw the MMAs of stage i - 5 complete.
  static constexpr int kStages = 3;
  static constexpr int kRawStages = 4;
  static constexpr int kGroupThreads = 256;  // one converter group
  static constexpr int kConvThreads = 2 * kGroupThreads;
  static constexpr int kChunks = kRawBytes / 16 / kGroupThreads;  // 16-byte chunks per thread and stage
  static constexpr int kEpiThreads = 128;
  static constexpr int kThreads = 736;
  static constexpr int kWarpW = 20;    // weight TMA
  static constexpr int kWarpMMA = 21;  // MMA issuer, TMEM owner
  static constexpr int kWarpX = 22;    // token-row TMA
  static constexpr int kTmemCols = 512;
  static constexpr int kMaxG = 256;
  static constexpr int kOffW = 0;
  static constexpr int kOffX = kOffW + kStages * kWBytes;
  static constexpr int kOffRaw = kOffX + kStages * kXBytes;
  static constexpr int kOffBar = kOffRaw + kRawStages * kRawBytes;
  static constexpr int kOffMisc = kOffBar + (2 * kRawStages + 3 * kStages + 8) * 8;
  static constexpr int kOffPrefix = kOffMisc + 64;                  // int[kMaxG + 1]
  static constexpr int kOffOffsets = kOffPrefix + (kMaxG + 1) * 4;  // int[kMaxG + 1]
  // int4: two slots of an item's group scales, 256 rows x up to 32 groups of bf16
  static constexpr int kScaleMaxGroups = 32;
  static constexpr int kScaleSlotBytes = WFMT == SB_W_INT4 ? kWRows * kScaleMaxGroups * 2 : 0;
  static constexpr int kOffScale = (kOffOffsets + (kMaxG + 1) * 4 + 127) / 128 * 128;  // 16-byte aligned copies
  // epilogue: per item the 256 weight rows' bias and fp8 scale, two buffers
  static constexpr int kOffEpi = kOffScale + 2 * kScaleSlotBytes;
  static constexpr int kEpiBytes = 2 * 2 * kWRows * 4;
  static constexpr int kSmemBytes = kOffEpi + kEpiBytes + 1024;
  static_assert(WFMT == SB_W_FP8 || WFMT == SB_W_INT4, "packed weight formats only");
  static_assert(EPI == SB_EPI_LINEAR || EPI == SB_EPI_GELU || EPI == SB_EPI_SWIGLU_IL, "one weight operand");
  static_assert(kChunks * 16 * kGroupThreads == kRawBytes, "whole chunks per thread");
  static_assert(kRawStages % 2 == 0, "raw slots must stay with one converter group");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
};

template <int WFMT, int EPI, bool kGather>
__global__ void __launch_bounds__(QCfg<WFMT, EPI>::kThreads, 1)
tc_gemm_qdec_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                    const __grid_constant__ CUtensorMap tmX128, const sb_grouped_gemm_args p) {
  using C = QCfg<WFMT, EPI>;
  constexpr int S = C::kStages, R = C::kRawStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* rfull = reinterpret_cast<uint64_t*>(smem + C::kOffBar);  // [R] packed weight tile landed
  uint64_t* rempty = rfull + R;                                      // [R] packed tile read by its converters
  uint64_t* xfull = rempty + R;                                      // [S] token rows landed
  uint64_t* conv = xfull + S;                                        // [S] bf16 weight tile written
  uint64_t* empty = conv + S;                                        // [S] stage's MMAs done
  uint64_t* acc_full = empty + S;                                    // [2]
  uint64_t* acc_empty = acc_full + 2;                                // [2]
  uint64_t* sfull = acc_empty + 2;                                   // [2] int4 scale slot landed
  uint64_t* sempty = sfull + 2;                                      // [2] int4 scale slot released
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  int* s_total = reinterpret_cast<int*>(smem + C::kOffMisc + 16);
  int* prefix = reinterpret_cast<int*>(smem + C::kOffPrefix);
  int* s_off = reinterpret_cast<int*>(smem + C::kOffOffsets);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.num_groups;
  const int f_tiles = (p.m_rows + C::kWRows - 1) / C::kWRows;
  const int fs = f_tiles * p.splits;  // items per token chunk: weight tiles x K splits
  const int nk = p.k / kTcBK / p.splits;
  // item t -> group g, token chunk nt, weight tile ft, K split ks (weight tile fastest)
  auto item = [&](int t, int& g, int& nt, int& ft, int& ks) {
    int fk;
    decode_tile(prefix, G, fs, t, g, nt, fk);
    ks = fk / f_tiles;
    ft = fk - ks * f_tiles;
  };
  // int4: an item's scales [256 rows x groups] by one bulk copy when the block
  // lies inside the scale matrix, fits a slot and starts 16-byte aligned
  // (producer and converters take the same decision per item)
  const int groups = WFMT == SB_W_INT4 ? static_cast<int>(p.lda / p.group_size) : 0;
  const __nv_bfloat16* scales = static_cast<const __nv_bfloat16*>(p.a_scale);
  auto bulk_scales = [&](int64_t arow0) {
    return WFMT == SB_W_INT4 && arow0 + C::kWRows <= p.a_rows_total && groups <= C::kScaleMaxGroups &&
           (reinterpret_cast<uintptr_t>(scales + arow0 * groups) & 15) == 0;
  };
  if (tid == 0) {
    for (int r = 0; r < R; ++r) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], C::kGroupThreads);
    }
    for (int s = 0; s < S; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&conv[s], C::kGroupThreads);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], C::kEpiThreads);
      mbar_init(&sfull[b], 1);
      mbar_init(&sempty[b], C::kConvThreads);
    }
    fence_barrier_init();
  }
  if (warp == C::kWarpW && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
    if (!kGather) tma_prefetch_desc(&tmX128);
  }
  pdl_wait();
  pdl_trigger();
  if (warp == 0) {
    // per-group items (128-token chunks x 256-row weight tiles) -> exclusive prefix
    int seen = 0;
    for (int base = 0; base < G; base += 32) {
      const int gi = base + lane;
      int items = 0;
      if (gi < G) {
        const int o0 = group_offset(p.offsets, gi, p.max_rows), o1 = group_offset(p.offsets, gi + 1, p.max_rows);
        s_off[gi] = o0;
        if (gi == G - 1) s_off[G] = o1;
        const int lo = min(o0, p.max_rows), hi = min(o1, p.max_rows);
        items = hi > lo ? (hi - lo + C::kTokM - 1) / C::kTokM * fs : 0;
      }
      int incl = items;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += t;
      }
      if (gi < G) prefix[gi] = seen + incl - items;
      seen += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      prefix[G] = seen;
      *s_total = seen;
    }
  }
  __syncthreads();
  const int total = *s_total;
  if (static_cast<int>(blockIdx.x) >= total) return;  // no item for this CTA
  const int my_items = (total - static_cast<int>(blockIdx.x) + gridDim.x - 1) / gridDim.x;

  if (warp == C::kWarpMMA) {
    tmem_alloc(s_tmem, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == C::kWarpW) {
    // ---------------------------------------------------------------- packed weight tiles (+ int4 scales)
    if (lane == 0) {
      int ri = 0, ub = 0;  // weight tiles and scale blocks issued
      bool ok = true;
      for (int j = 0; j < my_items && ok; ++j) {
        int g, nt, ft, ks;
        item(blockIdx.x + j * gridDim.x, g, nt, ft, ks);
        const int arow = static_cast<int>(static_cast<int64_t>(g) * p.a_group_rows + ft * C::kWRows);
        const int kb = ks * nk * kTcBK;
        if (bulk_scales(arow)) {
          const int sb = ub & 1;
          if (!mbar_wait(&sempty[sb], ((ub >> 1) & 1) ^ 1, p.status, SB_DEVERR_CONV_WAIT)) break;
          const uint32_t bytes = static_cast<uint32_t>(C::kWRows * groups * 2);
          mbar_expect_tx(&sfull[sb], bytes);
          bulk_load(smem + C::kOffScale + sb * C::kScaleSlotBytes, scales + static_cast<int64_t>(arow) * groups, bytes,
                    &sfull[sb]);
          ++ub;
        }
        for (int kk = 0; kk < nk; ++kk, ++ri) {
          const int k0 = kb + kk * kTcBK;
          const int r = ri % R;
          if (!mbar_wait(&rempty[r], ((ri / R) & 1) ^ 1, p.status, SB_DEVERR_CONV_WAIT)) { ok = false; break; }
          mbar_expect_tx(&rfull[r], C::kRawBytes);
          tma_load_2d(smem + C::kOffRaw + r * C::kRawBytes, &tmW, &rfull[r], WFMT == SB_W_INT4 ? k0 / 2 : k0, arow);
        }
      }
      for (int i = ri - R > 0 ? ri - R : 0; i < ri; ++i)  // drain
        if (!mbar_wait(&rfull[i % R], (i / R) & 1, p.status, SB_DEVERR_DRAIN)) break;
      for (int i = ub - 2 > 0 ? ub - 2 : 0; i < ub; ++i)
        if (!mbar_wait(&sfull[i & 1], (i >> 1) & 1, p.status, SB_DEVERR_DRAIN)) break;
    }
    __syncwarp();
  } else if (warp == C::kWarpX) {
    // ---------------------------------------------------------------- token rows
    int si = 0;
    bool ok = true;
    for (int j = 0; j < my_items && ok; ++j) {
      int g, nt, ft, ks;
      item(blockIdx.x + j * gridDim.x, g, nt, ft, ks);
      const int kb = ks * nk * kTcBK;
      const int n0 = s_off[g] + nt * C::kTokM;
      const int n_end = min(min(s_off[g + 1], p.max_rows), n0 + C::kTokM);
      // only the item's rows are fetched: 4-row gathers (one per lane), 16-row
      // boxes, or for more than 32 rows one 128-row box (the rows past the
      // item's end are other groups' or zero fill, and never stored)
      const bool wide = !kGather && n_end - n0 > 32;
      const int nb = kGather ? (n_end - n0 + 3) / 4 : (wide ? 1 : (n_end - n0 + 15) / 16);
      const uint32_t tx = kGather ? nb * 512u : (wide ? static_cast<uint32_t>(C::kXBytes) : nb * 2048u);
      int rix[4] = {0, 0, 0, 0};
      if (kGather && lane < nb) {
#pragma unroll
        for (int r = 0; r < 4; ++r) rix[r] = p.x_row_index[min(n0 + 4 * lane + r, n_end - 1)];
      }
      for (int kk = 0; kk < nk; ++kk, ++si) {
        const int s = si % S;
        bool w = true;
        if (lane == 0) {
          w = mbar_wait(&empty[s], ((si / S) & 1) ^ 1, p.status, SB_DEVERR_MMA_WAIT);
          if (w) mbar_expect_tx(&xfull[s], tx);
        }
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) { ok = false; break; }
        const int k0 = kb + kk * kTcBK;
        uint8_t* xdst = smem + C::kOffX + s * C::kXBytes;
        if (kGather) {
          __syncwarp();
          if (lane < nb) tma_gather4(xdst + lane * 512, &tmX, &xfull[s], k0, rix[0], rix[1], rix[2], rix[3]);
        } else if (lane == 0) {
          if (wide)
            tma_load_2d(xdst, &tmX128, &xfull[s], k0, n0);
          else
            for (int q = 0; q < nb; ++q) tma_load_2d(xdst + q * 2048, &tmX, &xfull[s], k0, n0 + 16 * q);
        }
      }
    }
    if (lane == 0)
      for (int i = si - S > 0 ? si - S : 0; i < si; ++i)  // drain
        if (!mbar_wait(&xfull[i % S], (i / S) & 1, p.status, SB_DEVERR_DRAIN)) break;
    __syncwarp();
  } else if (warp == C::kWarpMMA) {
    // ---------------------------------------------------------------- MMA issuer: D[token, weight row]
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(C::kTokM, C::kWRows);
      int si = 0;
      bool ok = true;
      for (int j = 0; j < my_items && ok; ++j) {
        const int buf = j & 1;
        if (!mbar_wait(&acc_empty[buf], ((j >> 1) & 1) ^ 1, p.status, SB_DEVERR_EPI_WAIT)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * C::kWRows;
        for (int kk = 0; kk < nk; ++kk, ++si) {
          const int s = si % S;
          const uint32_t ph = (si / S) & 1;
          ok = mbar_wait(&conv[s], ph, p.status, SB_DEVERR_CONV_WAIT) &&
               mbar_wait(&xfull[s], ph, p.status, SB_DEVERR_TMA_WAIT);
          if (!ok) break;
          tc_fence_after();
          const uint32_t x_base = smem_u32(smem + C::kOffX + s * C::kXBytes);
          const uint32_t w_base = smem_u32(smem + C::kOffW + s * C::kWBytes);
#pragma unroll
          for (int q = 0; q < kTcBK / 16; ++q)
            tc_mma_bf16(acc, smem_desc_k_sw128(x_base + q * 32), smem_desc_k_sw128(w_base + q * 32), idesc,
                        (kk > 0 || q > 0) ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        tc_commit(&acc_full[buf]);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- convert (warps 4-19)
    // Group cg = 0 / 1 converts the stages of even / odd global index.  Thread
    // gt of a group: int4 rows gt / 2 and 128 + gt / 2, 16-byte chunk gt % 2 of
    // 32 bytes; fp8 rows gt / 4 + 64 q (q < 4), chunk gt % 4 of 64 bytes.
    const int cg = (warp - 4) >> 3;
    const int gt = tid - 128 - cg * C::kGroupThreads;
    constexpr int kRowStep = WFMT == SB_W_INT4 ? 128 : 64;
    const int row0 = WFMT == SB_W_INT4 ? gt >> 1 : gt >> 2;
    const int c16 = WFMT == SB_W_INT4 ? gt & 1 : gt & 3;
    constexpr int kRowBytes = WFMT == SB_W_INT4 ? kTcBK / 2 : kTcBK;
    int ub = 0;
    bool ok = true;
    for (int j = 0; j < my_items && ok; ++j) {
      int g, nt, ft, ks;
      item(blockIdx.x + j * gridDim.x, g, nt, ft, ks);
      const int kb = ks * nk * kTcBK;
      const int64_t arow0 = static_cast<int64_t>(g) * p.a_group_rows + ft * C::kWRows;
      // int4 scales of this thread's rows: the item's bulk-copied block, else global memory
      const bool bulk = bulk_scales(arow0);
      const __nv_bfloat16* srow[C::kChunks];
      if (WFMT == SB_W_INT4) {
        if (bulk && !mbar_wait(&sfull[ub & 1], (ub >> 1) & 1, p.status, SB_DEVERR_TMA_WAIT)) break;
        const __nv_bfloat16* slot =
            reinterpret_cast<const __nv_bfloat16*>(smem + C::kOffScale + (ub & 1) * C::kScaleSlotBytes);
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c) {
          const int row = row0 + c * kRowStep;
          srow[c] = bulk ? slot + row * groups
                         : (arow0 + row < p.a_rows_total ? scales + (arow0 + row) * groups : nullptr);
        }
      }
      const int ci0 = j * nk;
      for (int kk = ((ci0 & 1) == cg) ? 0 : 1; kk < nk; kk += 2) {
        const int ci = ci0 + kk;
        const int r = ci % R, s = ci % S;
        const int k0 = kb + kk * kTcBK;
        __nv_bfloat16 sb[C::kChunks];
        if (WFMT == SB_W_INT4) {
#pragma unroll
          for (int c = 0; c < C::kChunks; ++c) sb[c] = srow[c] ? srow[c][k0 / p.group_size] : __float2bfloat16_rn(0.f);
        }
        if (!mbar_wait(&rfull[r], (ci / R) & 1, p.status, SB_DEVERR_TMA_WAIT)) { ok = false; break; }
        const uint8_t* raw = smem + C::kOffRaw + r * C::kRawBytes;
        uint4 v[C::kChunks];
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c)
          v[c] = *reinterpret_cast<const uint4*>(raw + (row0 + c * kRowStep) * kRowBytes + c16 * 16);
        // The packed bytes are in registers: the slot may refill.  The next
        // write into it is a TMA copy (async proxy), so the generic-proxy reads
        // above are ordered before it by a proxy fence ahead of the release.
        fence_proxy_async_smem();
        mbar_arrive(&rempty[r]);
        if (!mbar_wait(&empty[s], ((ci / S) & 1) ^ 1, p.status, SB_DEVERR_MMA_WAIT)) { ok = false; break; }
        uint8_t* dst = smem + C::kOffW + s * C::kWBytes;
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c) {
          if (WFMT == SB_W_INT4)
            convert_int4_chunk(v[c], sb[c], dst, row0 + c * kRowStep, c16);
          else
            convert_fp8_chunk(v[c], dst, row0 + c * kRowStep, c16);
        }
        fence_proxy_async_smem();
        mbar_arrive(&conv[s]);
      }
      if (bulk) {
        if (ok) {  // the item's scales are no longer read; the slot's next write is a bulk copy
          fence_proxy_async_smem();
          mbar_arrive(&sempty[ub & 1]);
        }
        ++ub;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 0-3)
    // Thread = one token row of the item (TMEM lane); its 256 columns are the
    // outputs of the item's 256 weight rows.  The rows' biases (and fp8
    // scales) are staged in shared memory once per item, two buffers deep.
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    constexpr int kVec = EPI == SB_EPI_LINEAR ? 4 : 8;  // elements per 16-byte store
    const bool vec_ok = (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 && p.ldo % kVec == 0 &&
                        (p.splits == 1 || p.split_stride % kVec == 0);
    for (int j = 0; j < my_items; ++j) {
      int g, nt, ft, ks;
      item(blockIdx.x + j * gridDim.x, g, nt, ft, ks);
      const int buf = j & 1;
      const int n0 = s_off[g] + nt * C::kTokM;
      const int tend = min(min(s_off[g + 1], p.max_rows), n0 + C::kTokM);
      const int tok = n0 + warp * 32 + lane;
      const bool tvalid = tok < tend;
      const float rs = (EPI == SB_EPI_LINEAR && p.row_scale && tvalid) ? p.row_scale[tok] : 1.f;
      const int wr0 = ft * C::kWRows;  // first weight row of the item within its group
      const int64_t arow0 = static_cast<int64_t>(g) * p.a_group_rows + wr0;
      const int wvalid = min(C::kWRows, p.m_rows - wr0);  // weight rows of this tile inside the group
      float* s_b = reinterpret_cast<float*>(smem + C::kOffEpi) + buf * 2 * C::kWRows;
      float* s_s = s_b + C::kWRows;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int wr = tid + h * 128;
        const bool wv = wr < wvalid;
        // K splits: the bias goes with split 0
        s_b[wr] = (p.bias && wv && ks == 0) ? p.bias[static_cast<int64_t>(g) * p.bias_group_stride + wr0 + wr] : 0.f;
        s_s[wr] = WFMT == SB_W_FP8 ? ((wv && arow0 + wr < p.a_rows_total)
                                          ? static_cast<const float*>(p.a_scale)[arow0 + wr] : 0.f)
                                   : 1.f;
      }
      bool ready = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (j >> 1) & 1, p.status, SB_DEVERR_EPI_WAIT));
      // one barrier of the four epilogue warps: the item's tables are written,
      // and all four take the same path if a wait gave up
      ready = named_bar_and(1, C::kEpiThreads, ready);
      tc_fence_after();
      if (!ready) break;
      const uint32_t acc_addr = lane_addr + buf * C::kWRows;
      if (__any_sync(0xffffffffu, tvalid)) {  // tcgen05.ld is warp-collective
        if constexpr (C::kIL) {
          // columns [gate 64 | up 64] per 128-row block: the features of block b
          // are (wr0 + 128 b) / 2 + i, i < 64
#pragma unroll 1
          for (int b = 0; b < 2; ++b) {
            if (b * 128 >= wvalid) break;
            const int64_t feat0 = (wr0 + b * 128) / 2;
#pragma unroll 1
            for (int c0 = 0; c0 < 64; c0 += 16) {
              float gv[16], uv[16], o[16];
              tmem_ld16x2(acc_addr + b * 128 + c0, acc_addr + b * 128 + 64 + c0, gv, uv);
              const int gr = b * 128 + c0, ur = gr + 64;
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                const float gate = silu_bf16out(gv[q] * s_s[gr + q] + s_b[gr + q]);
                o[q] = (uv[q] * s_s[ur + q] + s_b[ur + q]) * gate;
              }
              if (!tvalid) continue;
              __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(tok) * p.ldo + feat0 + c0;
              if (vec_ok) {
                uint32_t w[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  const __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * q], o[2 * q + 1]);
                  w[q] = *reinterpret_cast<const uint32_t*>(&h);
                }
                reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
                reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
              } else {
#pragma unroll
                for (int q = 0; q < 16; ++q) dst[q] = __float2bfloat16_rn(o[q]);
              }
            }
          }
        } else {
#pragma unroll 1
          for (int c0 = 0; c0 < C::kWRows; c0 += 32) {
            if (c0 >= wvalid) break;  // warp-uniform
            float va[16], vb[16];
            tmem_ld16x2(acc_addr + c0, acc_addr + c0 + 16, va, vb);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const float* v = hh ? vb : va;
              const int cc = c0 + 16 * hh;
              if (cc >= wvalid || !tvalid) continue;
              float o[16];
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                const float x = v[q] * s_s[cc + q] + s_b[cc + q];
                o[q] = EPI == SB_EPI_LINEAR ? x * rs : gelu_bf16out(x);
              }
              const int nv = min(16, wvalid - cc);
              const int64_t base = static_cast<int64_t>(ks) * p.split_stride + static_cast<int64_t>(tok) * p.ldo + wr0 + cc;
              if (EPI == SB_EPI_LINEAR) {
                float* dst = static_cast<float*>(p.out) + base;
                if (vec_ok && nv == 16) {
#pragma unroll
                  for (int q = 0; q < 4; ++q)
                    reinterpret_cast<float4*>(dst)[q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
                } else {
#pragma unroll
                  for (int q = 0; q < 16; ++q)
                    if (q < nv) dst[q] = o[q];
                }
              } else {
                __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.out) + base;
                if (vec_ok && nv == 16) {
                  uint32_t w[8];
#pragma unroll
                  for (int q = 0; q < 8; ++q) {
                    const __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * q], o[2 * q + 1]);
                    w[q] = *reinterpret_cast<const uint32_t*>(&h);
                  }
                  reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
                  reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
                } else {
#pragma unroll
                  for (int q = 0; q < 16; ++q)
                    if (q < nv) dst[q] = __float2bfloat16_rn(o[q]);
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == C::kWarpMMA) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ persistent CTA-pair GEMM
//
// The persistent schedule of the kernel above on CTA pairs (clusters of two):
// a pair computes a 256-feature x BN-token tile with tcgen05.mma.cta_group::2,
// each CTA holding 128 weight rows and BN/2 token rows of every K stage, so a
// CTA moves 32 KB of operands per 64-deep K step instead of 48 KB for the same
// work per SM.  The leader (cluster rank 0) issues the MMAs; commits arrive in
// both CTAs.  bf16 weights: each CTA's loads count on the leader's stage
// barrier.  fp8 / int4: loads count on the CTA's own barrier, its dequant warps
// convert and then arrive on the leader's conversion barrier.
// Warps as in the one-CTA kernel: 0-3, 6-9 epilogue, 4 TMA, 5 MMA, 10-13 dequant.
// Shared memory for the pair kernel's pipeline stages.
#ifndef SB_PAIR_STAGE_BUDGET
#define SB_PAIR_STAGE_BUDGET (200 * 1024)
#endif

template <int BN, int WFMT, int EPI>
struct PairCfg {
  static constexpr bool kGate = EPI == SB_EPI_SWIGLU;
  static constexpr bool kIL = EPI == SB_EPI_SWIGLU_IL;
  static constexpr bool kConvert = WFMT != SB_W_BF16;
  static constexpr int kBH = BN / 2;  // token rows of B per CTA
  static constexpr int kABytes = kTcBM * kTcBK * 2;
  static constexpr int kBBytes = kBH * kTcBK * 2;
  static constexpr int kRawBytes = WFMT == SB_W_FP8 ? kTcBM * kTcBK : (WFMT == SB_W_INT4 ? kTcBM * kTcBK / 2 : 0);
  static constexpr int kStageBytes = kABytes * (kGate ? 2 : 1) + kBBytes + kRawBytes * (kGate ? 2 : 1);
  // epilogue warps: 0-3 and 6-9, and for bf16 weights also 10-17 (four per
  // TMEM lane quarter, each a quarter of the tile's columns: the GELU
  // epilogue of short-K tiles would otherwise outlast the next tile's MMAs);
  // with fp8 / int4 weights warps 10-13 convert instead
  static constexpr int kEpiWarps = kConvert ? 8 : 16;
  static constexpr int kConvWarps = 4;
  static constexpr int kThreads = kConvert ? 448 : 576;
  // Output staging for the bulk (TMA) stores of the epilogue: 1 KB per
  // epilogue warp, a box of 32 features x kStoreRows tokens (fp32: 8, bf16: 16).
  // Interleaved SwiGLU: the gate warp of each (gate, up) warp pair hands
  // silu(gate) to the up warp through a 2 KB buffer; only up warps store.
  static constexpr int kOutBytes = EPI == SB_EPI_LINEAR ? 4 : 2;
  static constexpr int kStoreRows = 1024 / (32 * kOutBytes);
  static constexpr int kXBytes = kIL ? (kEpiWarps / 2) * 2048 : 0;
  static constexpr int kStagingBytes = (kIL ? kEpiWarps / 2 : kEpiWarps) * 1024 + kXBytes;
  static constexpr int kMaxG = 256;
  static constexpr int kFixedBytes = (3 * 8 + 4) * 8 + 64 + 2 * (kMaxG + 1) * 4 + 1024;
  static constexpr int kSmemMax = 227 * 1024;
  static constexpr int kBudget = (SB_PAIR_STAGE_BUDGET) < kSmemMax - kStagingBytes - kFixedBytes
                                     ? (SB_PAIR_STAGE_BUDGET) : kSmemMax - kStagingBytes - kFixedBytes;
  static constexpr int kStagesRaw = kBudget / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : (kStagesRaw < 2 ? 2 : kStagesRaw);
  static constexpr int kAccCols = BN * (kGate ? 2 : 1);
  static constexpr int kTmemCols = 2 * kAccCols;
  // B stages first: every operand read stays inside the allocation
  static constexpr int kOffB = 0;
  static constexpr int kOffA = kOffB + kStages * kBBytes;
  static constexpr int kOffG = kOffA + kStages * kABytes;
  static constexpr int kOffRaw = kOffG + (kGate ? kStages * kABytes : 0);
  static constexpr int kOffRawG = kOffRaw + kStages * kRawBytes;
  static constexpr int kOffOut = kOffRawG + (kGate ? kStages * kRawBytes : 0);
  static constexpr int kOffX = kOffOut + (kIL ? kEpiWarps / 2 : kEpiWarps) * 1024;
  static constexpr int kOffBar = kOffOut + kStagingBytes;
  static constexpr int kOffMisc = kOffBar + (3 * kStages + 4) * 8;
  static constexpr int kOffPrefix = kOffMisc + 64;
  static constexpr int kOffOffsets = kOffPrefix + (kMaxG + 1) * 4;
  static constexpr int kSmemBytes = kOffOffsets + (kMaxG + 1) * 4 + 1024;
  static_assert(kTmemCols <= 512, "two accumulators must fit the 512 TMEM columns");
  static_assert(kSmemBytes <= kSmemMax, "shared memory per CTA");
  static_assert(kBBytes % 1024 == 0 && kABytes % 1024 == 0, "1024-byte aligned swizzled stages");
  static_assert(kOffOut % 1024 == 0, "aligned output staging");
  static_assert(BN == 128 || BN == 256, "pair tiles are 128 or 256 tokens wide");
};

// tmO (when tma_out): the output [max_rows, m_rows] with a box of 32 features x
// kStoreRows tokens; full 16-token chunks of 32 valid features leave through it.
template <int BN, int WFMT, int EPI>
__global__ void __launch_bounds__(PairCfg<BN, WFMT, EPI>::kThreads, 1)
tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmG,
                    const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmO,
                    const sb_grouped_gemm_args p, const int tma_out) {
  using C = PairCfg<BN, WFMT, EPI>;
  constexpr int S = C::kStages;
  constexpr int kPairM = 2 * kTcBM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + S;
  uint64_t* conv = empty + S;
  uint64_t* acc_full = conv + S;       // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  int* prefix = reinterpret_cast<int*>(smem + C::kOffPrefix);
  int* s_off = reinterpret_cast<int*>(smem + C::kOffOffsets);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  const int G = p.num_groups;
  const int m_tiles = (p.m_rows + kPairM - 1) / kPairM;
  const int nk = p.k / kTcBK;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 2 * C::kConvWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * C::kEpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (C::kGate) tma_prefetch_desc(&tmG);
  }
  pdl_wait();
  pdl_trigger();
  if (warp == 0) {
    int seen = 0;
    for (int base = 0; base < G; base += 32) {
      const int gi = base + lane;
      int tiles = 0;
      if (gi < G) {
        const int o0 = group_offset(p.offsets, gi, p.max_rows), o1 = group_offset(p.offsets, gi + 1, p.max_rows);
        s_off[gi] = o0;
        if (gi == G - 1) s_off[G] = o1;
        const int lo = min(o0, p.max_rows), hi = min(o1, p.max_rows);
        tiles = hi > lo ? (hi - lo + BN - 1) / BN * m_tiles : 0;
      }
      int incl = tiles;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += t;
      }
      if (gi < G) prefix[gi] = seen + incl - tiles;
      seen += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) prefix[G] = seen;
  }
  // both CTAs' barriers initialised (and this CTA's tile table written) before
  // any CTA of the pair signals the other
  __syncwarp();
  cluster_sync();
  const int total = prefix[G];
  if (pair >= total) return;  // both CTAs of the pair leave: nothing to do
  const int my_tiles = (total - pair + npairs - 1) / npairs;
  const uint32_t full_lead = mapa_shared(smem_u32(full), 0);
  const uint32_t conv_lead = mapa_shared(smem_u32(conv), 0);
  const uint32_t acc_empty_lead = mapa_shared(smem_u32(acc_empty), 0);

  if (warp == 5) {
    tmem_alloc_pair(s_tmem, C::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 4) {
    // ---------------------------------------------------------------- producer (both CTAs)
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int j = 0; j < my_tiles && ok; ++j) {
        int g, nt, mt;
        decode_tile(prefix, G, m_tiles, pair + j * npairs, g, nt, mt);
        const int arow = static_cast<int>(static_cast<int64_t>(g) * p.a_group_rows) + mt * kPairM + static_cast<int>(rank) * kTcBM;
        // each CTA holds half of the tile's MMA columns: with a short last
        // tile (tile_mma_n < BN) CTA 1's half starts at the narrower midpoint
        const int tile_n0 = s_off[g] + nt * BN;
        const int tile_end = min(min(s_off[g + 1], p.max_rows), tile_n0 + BN);
        const int nrow = tile_n0 + static_cast<int>(rank) * (tile_mma_n<BN>(tile_end - tile_n0) / 2);
        for (int kk = 0; kk < nk; ++kk, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, p.status, SB_DEVERR_MMA_WAIT)) { ok = false; break; }
          const int k0 = kk * kTcBK;
          if (C::kConvert) {
            // raw weights + this CTA's token rows on its own barrier (dequant warps wait on it)
            mbar_expect_tx(&full[s], C::kRawBytes * (C::kGate ? 2 : 1) + C::kBBytes);
            const int acol = WFMT == SB_W_INT4 ? k0 / 2 : k0;
            tma_load_2d(smem + C::kOffRaw + s * C::kRawBytes, &tmA, &full[s], acol, arow);
            if (C::kGate) tma_load_2d(smem + C::kOffRawG + s * C::kRawBytes, &tmG, &full[s], acol, arow);
            tma_load_2d(smem + C::kOffB + s * C::kBBytes, &tmB, &full[s], k0, nrow);
          } else {
            // both CTAs' bytes count on the leader's barrier; the leader arrives once
            if (leader) mbar_expect_tx(&full[s], 2 * (C::kABytes * (C::kGate ? 2 : 1) + C::kBBytes));
            const uint32_t bar = full_lead + 8u * s;
            tma_load_2d_pair(smem + C::kOffA + s * C::kABytes, &tmA, bar, k0, arow);
            if (C::kGate) tma_load_2d_pair(smem + C::kOffG + s * C::kABytes, &tmG, bar, k0, arow);
            tma_load_2d_pair(smem + C::kOffB + s * C::kBBytes, &tmB, bar, k0, nrow);
          }
        }
      }
      // Drain: the MMAs released every stage (all copies landed, all commit
      // arrivals on this CTA's barriers done) before the CTA may exit.
      for (int i = it - S > 0 ? it - S : 0; i < it; ++i)
        if (!mbar_wait(&empty[i % S], (i / S) & 1, p.status, SB_DEVERR_DRAIN)) break;
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer (leader)
    if (leader && lane == 0) {
      int it = 0;
      bool ok = true;
      for (int j = 0; j < my_tiles && ok; ++j) {
        const int buf = j & 1;
        int g, nt, mt;
        decode_tile(prefix, G, m_tiles, pair + j * npairs, g, nt, mt);
        const int tile_n0 = s_off[g] + nt * BN;
        const int tile_end = min(min(s_off[g + 1], p.max_rows), tile_n0 + BN);
        const uint32_t idesc = idesc_bf16_f32(kPairM, tile_mma_n<BN>(tile_end - tile_n0));
        if (!mbar_wait_cluster(&acc_empty[buf], ((j >> 1) & 1) ^ 1, p.status, SB_DEVERR_EPI_WAIT)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * C::kAccCols;
        for (int kk = 0; kk < nk; ++kk, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          ok = C::kConvert ? mbar_wait_cluster(&conv[s], ph, p.status, SB_DEVERR_CONV_WAIT)
                           : mbar_wait(&full[s], ph, p.status, SB_DEVERR_TMA_WAIT);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + C::kOffA + s * C::kABytes);
          const uint32_t g_base = smem_u32(smem + C::kOffG + s * C::kABytes);
          const uint32_t b_base = smem_u32(smem + C::kOffB + s * C::kBBytes);
#pragma unroll
          for (int q = 0; q < kTcBK / 16; ++q) {
            const uint64_t bdesc = smem_desc_k_sw128(b_base + q * 32);
            const uint32_t accum = (kk > 0 || q > 0) ? 1u : 0u;
            tc_mma_bf16_pair(acc, smem_desc_k_sw128(a_base + q * 32), bdesc, idesc, accum);
            if (C::kGate) tc_mma_bf16_pair(acc + BN, smem_desc_k_sw128(g_base + q * 32), bdesc, idesc, accum);
          }
          tc_commit_pair(&empty[s]);
        }
        tc_commit_pair(&acc_full[buf]);
      }
    }
    __syncwarp();
  } else if (C::kConvert && warp >= 10) {
    // ---------------------------------------------------------------- dequant (fp8 / int4, both CTAs)
    {
      const int ctid = tid - 320;
      int it = 0;
      for (int j = 0; j < my_tiles; ++j) {
        int g, nt, mt;
        decode_tile(prefix, G, m_tiles, pair + j * npairs, g, nt, mt);
        const int64_t arow0 = static_cast<int64_t>(g) * p.a_group_rows + mt * kPairM + rank * kTcBM;
        bool ok = true;
        for (int kk = 0; kk < nk; ++kk, ++it) {
          const int s = it % S;
          if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (it / S) & 1, p.status, SB_DEVERR_TMA_WAIT))) {
            ok = false;
            break;
          }
          const int k0 = kk * kTcBK;
          convert_tile<WFMT>(smem + C::kOffRaw + s * C::kRawBytes, smem + C::kOffA + s * C::kABytes, p,
                             p.a_scale, arow0, k0, ctid);
          if (C::kGate)
            convert_tile<WFMT>(smem + C::kOffRawG + s * C::kRawBytes, smem + C::kOffG + s * C::kABytes, p,
                               p.a_gate_scale, arow0, k0, ctid);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(conv_lead + 8u * s);
        }
        if (!ok) break;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    // warp w reads TMEM lane quarter w % 4; its ordinal / 4 picks the column part
    constexpr int kParts = C::kEpiWarps / 4;
    constexpr int HB = BN / kParts;
    const int quarter = warp & 3;
    const int ord = warp < 4 ? warp : warp - 2;  // 0 .. kEpiWarps - 1
    const int half = ord >> 2;                   // column part
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + half * HB;
    uint8_t* stage_out = smem + C::kOffOut + ord * 1024;
    for (int j = 0; j < my_tiles; ++j) {
      int g, nt, mt;
      decode_tile(prefix, G, m_tiles, pair + j * npairs, g, nt, mt);
      const int buf = j & 1;
      const int m = mt * kPairM + static_cast<int>(rank) * kTcBM + quarter * 32 + lane;
      const int64_t arow = static_cast<int64_t>(g) * p.a_group_rows + m;
      const bool mvalid = m < p.m_rows && arow < p.a_rows_total;
      const float sa = ((WFMT == SB_W_FP8 || (WFMT == SB_W_BF16 && p.a_scale)) && mvalid) ? static_cast<const float*>(p.a_scale)[arow] : 1.f;
      const float sg = (C::kGate && (WFMT == SB_W_FP8 || (WFMT == SB_W_BF16 && p.a_gate_scale)) && mvalid) ? static_cast<const float*>(p.a_gate_scale)[arow] : 1.f;
      const float bias = (p.bias && mvalid) ? p.bias[static_cast<int64_t>(g) * p.bias_group_stride + m] : 0.f;
      const float bgate = (C::kGate && p.bias_gate && mvalid) ? p.bias_gate[static_cast<int64_t>(g) * p.bias_group_stride + m] : 0.f;
      const int tn0 = s_off[g] + nt * BN + half * HB;
      const int tend = min(min(s_off[g] + nt * BN + BN, s_off[g + 1]), p.max_rows);
      float rsv[HB / 32];
#pragma unroll
      for (int i = 0; i < HB / 32; ++i) {
        const int r = tn0 + i * 32 + lane;
        rsv[i] = (EPI == SB_EPI_LINEAR && p.row_scale && r < tend) ? p.row_scale[r] : 1.f;
      }
      bool ready = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (j >> 1) & 1, p.status, SB_DEVERR_EPI_WAIT));
      // interleaved SwiGLU: quarters 0-1 hold gate rows, 2-3 the up rows of the
      // same features; warp pair (quarter q, q + 2) of each column part
      const int xpair = half * 2 + (quarter & 1);
      if (C::kIL) ready = named_bar_and(1 + xpair, 64, ready);
      tc_fence_after();
      if (!ready) break;
      const uint32_t acc_addr = lane_addr + buf * C::kAccCols;
      // bulk stores need all 32 features of the warp in range
      const bool bulk = tma_out && __all_sync(0xffffffffu, mvalid);
#pragma unroll
      for (int c0 = 0; c0 < HB; c0 += 16) {
        if (tn0 + c0 >= tend) break;  // warp-uniform
        float v[16], vg[16], o[16];
        tmem_ld16(acc_addr + c0, v);
        if (C::kGate) tmem_ld16(acc_addr + BN + c0, vg);
        if constexpr (C::kIL) {
          float* xb = reinterpret_cast<float*>(smem + C::kOffX) + xpair * 512;
          if (quarter < 2) {
#pragma unroll
            for (int q = 0; q < 16; ++q) xb[q * 32 + lane] = silu_bf16out(v[q] * sa + bias);
            named_bar_sync(1 + xpair, 64);
            named_bar_sync(1 + xpair, 64);
            continue;
          }
#pragma unroll
          for (int q = 0; q < 16; ++q) o[q] = v[q] * sa + bias;
          named_bar_sync(1 + xpair, 64);
#pragma unroll
          for (int q = 0; q < 16; ++q) o[q] *= xb[q * 32 + lane];
          named_bar_sync(1 + xpair, 64);
          const int fo0 = (mt * kPairM + static_cast<int>(rank) * kTcBM) / 2 + (quarter - 2) * 32;  // lane 0's feature
          const int nvalid = tend - (tn0 + c0);
          if (bulk && nvalid >= 16) {
            uint8_t* so = smem + C::kOffOut + xpair * 1024;
            if (lane == 0) tma_store_wait_read();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 16; ++q) reinterpret_cast<__nv_bfloat16*>(so)[q * 32 + lane] = __float2bfloat16_rn(o[q]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) tma_store_2d(&tmO, so, fo0, tn0 + c0);
            continue;
          }
          if (!mvalid) continue;
          const int64_t base = static_cast<int64_t>(tn0 + c0) * p.ldo + fo0 + lane;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            if (nvalid < 16 && q >= nvalid) break;
            static_cast<__nv_bfloat16*>(p.out)[base + static_cast<int64_t>(q) * p.ldo] = __float2bfloat16_rn(o[q]);
          }
          continue;
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float x = v[q] * sa + bias;
          if (EPI == SB_EPI_LINEAR)
            o[q] = x * __shfl_sync(0xffffffffu, rsv[(c0 + q) >> 5], (c0 + q) & 31);
          else if (EPI == SB_EPI_GELU)
            o[q] = gelu_bf16out(x);
          else
            o[q] = silu_bf16out(vg[q] * sg + bgate) * x;
        }
        const int nvalid = tend - (tn0 + c0);
        if (bulk && nvalid >= 16) {
          // a whole chunk: 32 features x 16 tokens through the staging box
          // (token-major, as the output rows), then one bulk store per box
#pragma unroll
          for (int h = 0; h < 16 / C::kStoreRows; ++h) {
            if (lane == 0) tma_store_wait_read();  // the previous box has left the buffer
            __syncwarp();
#pragma unroll
            for (int q = 0; q < C::kStoreRows; ++q) {
              if (EPI == SB_EPI_LINEAR)
                reinterpret_cast<float*>(stage_out)[q * 32 + lane] = o[h * C::kStoreRows + q];
              else
                reinterpret_cast<__nv_bfloat16*>(stage_out)[q * 32 + lane] =
                    __float2bfloat16_rn(o[h * C::kStoreRows + q]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) tma_store_2d(&tmO, stage_out, m - lane, tn0 + c0 + h * C::kStoreRows);
          }
          continue;
        }
        if (!mvalid) continue;
        const int64_t base = static_cast<int64_t>(tn0 + c0) * p.ldo + m;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if (nvalid < 16 && q >= nvalid) break;
          if (EPI == SB_EPI_LINEAR)
            static_cast<float*>(p.out)[base + static_cast<int64_t>(q) * p.ldo] = o[q];
          else
            static_cast<__nv_bfloat16*>(p.out)[base + static_cast<int64_t>(q) * p.ldo] = __float2bfloat16_rn(o[q]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_lead + 8u * buf);
    }
    if (lane == 0) tma_store_wait_all();  // every bulk store complete before the CTA leaves
    __syncwarp();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the other may still touch its shared memory
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D tensor map: inner extent `cols` elements, `rows` rows, row pitch in bytes.
static bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t cols, uint64_t rows,
                     uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool weight_map(CUtensorMap* m, const sb_grouped_gemm_args& a, const void* base) {
  if (a.wfmt == SB_W_BF16)
    return make_map(m, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.lda, a.a_rows_total, a.lda * 2, kTcBK, kTcBM,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (a.wfmt == SB_W_FP8)
    return make_map(m, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.lda, a.a_rows_total, a.lda, kTcBK, kTcBM,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
  return make_map(m, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.lda / 2, a.a_rows_total, a.lda / 2, kTcBK / 2, kTcBM,
                  CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool tcgen05_supported(const sb_grouped_gemm_args& a) {
  if (a.act_dtype != SB_BF16) return false;
  if (a.wfmt != SB_W_BF16 && a.wfmt != SB_W_FP8 && a.wfmt != SB_W_INT4) return false;
  if (a.splits <= 0 || a.k % (kTcBK * a.splits)) return false;
  if (a.wfmt == SB_W_INT4 && (a.group_size <= 0 || a.group_size % kTcBK || a.lda % a.group_size)) return false;
  if (a.ldx % 8 || (a.wfmt == SB_W_BF16 && a.lda % 8) || (a.wfmt != SB_W_BF16 && a.lda % 32)) return false;
  if (reinterpret_cast<uintptr_t>(a.a) % 16 || reinterpret_cast<uintptr_t>(a.x) % 16) return false;
  if (a.epilogue == SB_EPI_SWIGLU && (!a.a_gate || reinterpret_cast<uintptr_t>(a.a_gate) % 16)) return false;
  if (a.epilogue == SB_EPI_SWIGLU_IL && a.m_rows % kTcBM) return false;  // whole 64-feature blocks
  if (a.a_rows_total > 0x7fffffffLL || a.max_rows <= 0) return false;
  if (a.x_row_index && (tc_tile_n(a) > 64 || a.x_rows <= 0)) return false;
  return current_cc_major() == 10;
}

template <int BN, int WFMT, int EPI, bool kFixed, bool kGather>
static int launch_tc(const sb_grouped_gemm_args& a, cudaStream_t st) {
  using C = TcCfg<BN, WFMT, EPI, kFixed>;
  auto kern = tc_gemm_kernel<BN, WFMT, EPI, kFixed, kGather>;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return cuda_status(e);
    configured_device = dev;
  }
  CUtensorMap ma, mg, mb;
  if (!weight_map(&ma, a, a.a)) return SB_ERR_UNSUPPORTED;
  mg = ma;
  if (C::kGate && !weight_map(&mg, a, a.a_gate)) return SB_ERR_UNSUPPORTED;
  bool ok_b;
  if (kGather)  // source rows: a one-row box of 64 elements (128 bytes), 128-byte swizzle
    ok_b = make_map(&mb, a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.k, a.x_rows, a.ldx * 2, kTcBK, 1,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  else  // fixed-group schedule: 16-row boxes, only as many as the tile's valid rows need
    ok_b = make_map(&mb, a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.k, a.max_rows, a.ldx * 2, kTcBK,
                    kFixed ? 16 : BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok_b) return SB_ERR_UNSUPPORTED;
  const int m_tiles = (a.m_rows + kTcBM - 1) / kTcBM;
  const dim3 grid(m_tiles, kFixed ? a.num_groups : (a.max_rows + BN - 1) / BN + a.num_groups, a.splits);
  return launch(kern, grid, dim3(kTcThreads), C::kSmemBytes, st, ma, mg, mb, a);
}

constexpr int kPersistentMaxGroups = 256;

// SPIDER_B200_PERSISTENT=0 selects the one-tile-per-CTA kernel for large tiles
// (for comparisons); the default is the persistent kernel.
static bool use_persistent(const sb_grouped_gemm_args& a) {
  static const bool enabled = [] {
    const char* e = std::getenv("SPIDER_B200_PERSISTENT");
    return !(e && e[0] == '0');
  }();
  return enabled && a.splits == 1 && a.num_groups <= kPersistentMaxGroups;
}

template <int BN, int WFMT, int EPI>
static int launch_persistent(const sb_grouped_gemm_args& a, cudaStream_t st) {
  using C = PCfg<BN, WFMT, EPI>;
  auto kern = tc_gemm_persistent_kernel<BN, WFMT, EPI>;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    configured_device = dev;
  }
  static_assert(C::kMaxG == kPersistentMaxGroups, "tile table size");
  if (a.num_groups > C::kMaxG || a.splits != 1) return SB_ERR_UNSUPPORTED;
  CUtensorMap ma, mg, mb;
  if (!weight_map(&ma, a, a.a)) return SB_ERR_UNSUPPORTED;
  mg = ma;
  if (C::kGate && !weight_map(&mg, a, a.a_gate)) return SB_ERR_UNSUPPORTED;
  if (!make_map(&mb, a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.k, a.max_rows, a.ldx * 2, kTcBK, BN,
                CU_TENSOR_MAP_SWIZZLE_128B))
    return SB_ERR_UNSUPPORTED;
  const int m_tiles = (a.m_rows + kTcBM - 1) / kTcBM;
  const int64_t bound = static_cast<int64_t>(m_tiles) * ((a.max_rows + BN - 1) / BN + a.num_groups);
  const int sms = current_sm_count();
  const int grid = static_cast<int>(bound < sms ? bound : sms);
  return launch(kern, dim3(grid), dim3(C::kThreads), C::kSmemBytes, st, ma, mg, mb, a);
}

// SPIDER_B200_QDEC=0 keeps quantised decode GEMMs on the tiled kernels (for comparisons).
bool tc_qdec(const sb_grouped_gemm_args& a) {
  static const bool enabled = [] {
    const char* e = std::getenv("SPIDER_B200_QDEC");
    return !(e && e[0] == '0');
  }();
  // bf16 decode stays on the fixed-group kernel (measured faster: no
  // conversion to share, several CTAs per SM stream the weights)
  if (!enabled || (a.wfmt != SB_W_FP8 && a.wfmt != SB_W_INT4)) return false;
  if (a.num_groups > kPersistentMaxGroups || a.epilogue == SB_EPI_SWIGLU) return false;
  if (a.splits != 1 && a.epilogue != SB_EPI_LINEAR) return false;
  if (a.x_row_index && a.x_rows <= 0) return false;
  // decode batches: the expected rows per group are few (the tiled kernels'
  // column tile would be at most 64)
  const int hint = a.rows_hint > 0 ? a.rows_hint : a.max_rows;
  return (hint + a.num_groups - 1) / a.num_groups <= 64;
}

template <int WFMT, int EPI, bool kGather>
static int launch_qdec(const sb_grouped_gemm_args& a, cudaStream_t st) {
  using C = QCfg<WFMT, EPI>;
  auto kern = tc_gemm_qdec_kernel<WFMT, EPI, kGather>;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    configured_device = dev;
  }
  static_assert(C::kMaxG == kPersistentMaxGroups, "prefix table size");
  if (a.num_groups > C::kMaxG || a.splits < 1 || (a.splits != 1 && EPI != SB_EPI_LINEAR)) return SB_ERR_UNSUPPORTED;
  // weights: 256-row boxes of one K step (packed bytes); tokens: 16-row boxes or one-row gathers
  CUtensorMap mw, mx;
  const bool ok_w =
      WFMT == SB_W_FP8
          ? make_map(&mw, a.a, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.lda, a.a_rows_total, a.lda, kTcBK, C::kWRows,
                     CU_TENSOR_MAP_SWIZZLE_NONE)
          : make_map(&mw, a.a, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.lda / 2, a.a_rows_total, a.lda / 2, kTcBK / 2,
                     C::kWRows, CU_TENSOR_MAP_SWIZZLE_NONE);
  CUtensorMap mx128;
  const bool ok_x =
      kGather ? make_map(&mx, a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.k, a.x_rows, a.ldx * 2, kTcBK, 1,
                         CU_TENSOR_MAP_SWIZZLE_128B)
              : make_map(&mx, a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.k, a.max_rows, a.ldx * 2, kTcBK, 16,
                         CU_TENSOR_MAP_SWIZZLE_128B) &&
                    make_map(&mx128, a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.k, a.max_rows, a.ldx * 2, kTcBK,
                             C::kTokM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok_w || !ok_x) return SB_ERR_UNSUPPORTED;
  if (kGather) mx128 = mx;  // unused
  const int f_tiles = (a.m_rows + C::kWRows - 1) / C::kWRows;
  const int64_t bound =
      static_cast<int64_t>(f_tiles) * a.splits * ((a.max_rows + C::kTokM - 1) / C::kTokM + a.num_groups);
  const int sms = current_sm_count();
  const int grid = static_cast<int>(bound < sms ? bound : sms);
  return launch(kern, dim3(grid), dim3(C::kThreads), C::kSmemBytes, st, mw, mx, mx128, a);
}

template <int WFMT>
static int launch_qdec_epi(const sb_grouped_gemm_args& a, cudaStream_t st) {
  const bool g = a.x_row_index != nullptr;
  switch (a.epilogue) {
    case SB_EPI_LINEAR:
      return g ? launch_qdec<WFMT, SB_EPI_LINEAR, true>(a, st) : launch_qdec<WFMT, SB_EPI_LINEAR, false>(a, st);
    case SB_EPI_GELU:
      return g ? launch_qdec<WFMT, SB_EPI_GELU, true>(a, st) : launch_qdec<WFMT, SB_EPI_GELU, false>(a, st);
    case SB_EPI_SWIGLU_IL:
      return g ? launch_qdec<WFMT, SB_EPI_SWIGLU_IL, true>(a, st) : launch_qdec<WFMT, SB_EPI_SWIGLU_IL, false>(a, st);
    default: return SB_ERR_UNSUPPORTED;
  }
}

// SPIDER_B200_TMA_STORE=0 makes the large-tile epilogues store element by
// element instead of through shared memory and bulk tensor stores (for comparisons).
static bool use_tma_out() {
  static const bool enabled = [] {
    const char* e = std::getenv("SPIDER_B200_TMA_STORE");
    return !(e && e[0] == '0');
  }();
  return enabled;
}

// SPIDER_B200_PAIR=0 keeps large tiles on one-CTA tiles (for comparisons).
static bool use_pair(const sb_grouped_gemm_args& a) {
  static const bool enabled = [] {
    const char* e = std::getenv("SPIDER_B200_PAIR");
    return !(e && e[0] == '0');
  }();
  // fp8 / int4 weights stay on one-CTA tiles: their dequant-then-signal path
  // measured slower on pairs than the one-CTA kernel.  So do narrow weight
  // matrices (fewer than two 256-row pair tiles, as the dense routing
  // logits' 272 rows): the pair's second tile would be mostly empty rows.
  return enabled && a.m_rows >= 4 * kTcBM && a.wfmt == SB_W_BF16;
}

template <int BN, int WFMT, int EPI>
static int launch_pair(const sb_grouped_gemm_args& a, cudaStream_t st) {
  using C = PairCfg<BN, WFMT, EPI>;
  static_assert(C::kMaxG == kPersistentMaxGroups, "tile table size");
  auto kern = tc_gemm_pair_kernel<BN, WFMT, EPI>;
  static int configured_device = -1;
  static int max_pairs = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cfg.attrs = attr;
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    cfg.gridDim = dim3(2 * current_sm_count());
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = current_sm_count() / 2;
    }
    max_pairs = n;
    configured_device = dev;
  }
  if (a.num_groups > C::kMaxG || a.splits != 1) return SB_ERR_UNSUPPORTED;
  CUtensorMap ma, mg, mb;
  if (!weight_map(&ma, a, a.a)) return SB_ERR_UNSUPPORTED;
  mg = ma;
  if (C::kGate && !weight_map(&mg, a, a.a_gate)) return SB_ERR_UNSUPPORTED;
  if (!make_map(&mb, a.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.k, a.max_rows, a.ldx * 2, kTcBK, C::kBH,
                CU_TENSOR_MAP_SWIZZLE_128B))
    return SB_ERR_UNSUPPORTED;
  // The output as a tensor for the epilogue's bulk stores: [max_rows, m_rows]
  // with row pitch ldo (fp32 for LINEAR, else bf16); without one (an
  // unaligned output) every element is stored by the epilogue threads.
  CUtensorMap mo = mb;
  const int out_cols = C::kIL ? a.m_rows / 2 : a.m_rows;  // interleaved SwiGLU: two rows per feature
  const int tma_out = use_tma_out() && out_cols >= 32 &&
                      make_map(&mo, a.out, EPI == SB_EPI_LINEAR ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                                : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                               out_cols, a.max_rows, a.ldo * C::kOutBytes, 32, C::kStoreRows,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
  const int m_tiles = (a.m_rows + 2 * kTcBM - 1) / (2 * kTcBM);
  const int64_t bound = static_cast<int64_t>(m_tiles) * ((a.max_rows + BN - 1) / BN + a.num_groups);
  const int pairs = static_cast<int>(bound < max_pairs ? bound : max_pairs);
  cfg.gridDim = dim3(2 * pairs);
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  note_launch();
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, ma, mg, mb, mo, a, tma_out));
}

template <int BN, int WFMT, int EPI>
static int launch_modes(const sb_grouped_gemm_args& a, cudaStream_t st) {
  const bool g = a.x_row_index != nullptr;
  if (tc_fixed_groups(a))
    return g ? launch_tc<BN, WFMT, EPI, true, true>(a, st) : launch_tc<BN, WFMT, EPI, true, false>(a, st);
  return g ? launch_tc<BN, WFMT, EPI, false, true>(a, st) : launch_tc<BN, WFMT, EPI, false, false>(a, st);
}

template <int WFMT, int EPI>
static int launch_bn(const sb_grouped_gemm_args& a, cudaStream_t st, int bn) {
  const bool g = a.x_row_index != nullptr;
  switch (bn) {
    case 16: return launch_modes<16, WFMT, EPI>(a, st);
    case 32: return launch_modes<32, WFMT, EPI>(a, st);
    case 64: return launch_modes<64, WFMT, EPI>(a, st);
    // Large tiles: the persistent kernel (two TMEM accumulators; SwiGLU's two
    // accumulator sets fit only at 128 columns) unless the problem is K-split
    // or has more groups than its tile table holds.
    case 128:
      if (g) return SB_ERR_UNSUPPORTED;
      if (!use_persistent(a)) return launch_tc<128, WFMT, EPI, false, false>(a, st);
      if (use_pair(a)) return launch_pair<128, WFMT, EPI>(a, st);
      return launch_persistent<128, WFMT, EPI>(a, st);
    default:
      if (g) return SB_ERR_UNSUPPORTED;
      if (!use_persistent(a)) return launch_tc<256, WFMT, EPI, false, false>(a, st);
      if constexpr (EPI == SB_EPI_SWIGLU) {
        if (use_pair(a)) return launch_pair<128, WFMT, EPI>(a, st);
        return launch_persistent<128, WFMT, EPI>(a, st);
      } else {
        if (use_pair(a)) return launch_pair<256, WFMT, EPI>(a, st);
        return launch_persistent<256, WFMT, EPI>(a, st);
      }
  }
}

template <int WFMT>
static int launch_epi(const sb_grouped_gemm_args& a, cudaStream_t st, int bn) {
  switch (a.epilogue) {
    case SB_EPI_LINEAR: return launch_bn<WFMT, SB_EPI_LINEAR>(a, st, bn);
    case SB_EPI_GELU: return launch_bn<WFMT, SB_EPI_GELU>(a, st, bn);
    case SB_EPI_SWIGLU_IL: return launch_bn<WFMT, SB_EPI_SWIGLU_IL>(a, st, bn);
    default: return launch_bn<WFMT, SB_EPI_SWIGLU>(a, st, bn);
  }
}

// Fixed-group schedule when the caller expects every group's rows to fit one
// tile of <= 64 columns (each CTA then streams its weights once; a group with
// more rows is still covered: its CTA loops over the row tiles).
bool tc_fixed_groups(const sb_grouped_gemm_args& a) {
  return a.group_rows_bound > 0 && a.group_rows_bound <= 64;
}

// Column tile: the bound rounded up to 16 on the fixed-group schedule,
// otherwise the smallest of 16..256 that covers the expected rows per group.
int tc_tile_n(const sb_grouped_gemm_args& a) {
  if (tc_fixed_groups(a)) return a.group_rows_bound <= 16 ? 16 : (a.group_rows_bound <= 32 ? 32 : 64);
  const int hint = a.rows_hint > 0 ? a.rows_hint : a.max_rows;
  const int per_group = (hint + a.num_groups - 1) / a.num_groups;
  if (per_group <= 16) return 16;
  if (per_group <= 32) return 32;
  if (per_group <= 64) return 64;
  if (per_group <= 128) return 128;
  return 256;
}

// fp8 e4m3 / packed int4 weights [rows, k] -> bf16 [rows, k]: e4m3 exactly
// (its per-row scale stays with the GEMM epilogue), int4 as bf16(q * s) with
// the bf16 group scale -- the values convert_tile produces in shared memory.
// One thread per 16 source bytes.
__global__ void __launch_bounds__(256)
dequant_bf16_kernel(const uint8_t* __restrict__ q, int wfmt, const __nv_bfloat16* __restrict__ scales, int group_size,
                    int64_t rows, int64_t k, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t row_bytes = wfmt == SB_W_FP8 ? k : k / 2;
  const int64_t chunks = rows * (row_bytes / 16);
  const int64_t groups = wfmt == SB_W_INT4 ? k / group_size : 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < chunks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / (row_bytes / 16), cb = (i - r * (row_bytes / 16)) * 16;  // row, byte offset in the row
    const uint4 v = *reinterpret_cast<const uint4*>(q + r * row_bytes + cb);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
    if (wfmt == SB_W_FP8) {
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
            static_cast<__nv_fp8x2_storage_t>(b[2 * j] | (b[2 * j + 1] << 8)), __NV_E4M3);
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
        const __nv_bfloat162 bb = __floats2bfloat162_rn(f.x, f.y);
        o[j] = *reinterpret_cast<const uint32_t*>(&bb);
      }
      uint4* dst = reinterpret_cast<uint4*>(out + r * k + cb);
      dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
      dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    } else {
      const int64_t k0 = cb * 2;  // first weight of the chunk (32 weights)
      const float s = __bfloat162float(scales[r * groups + k0 / group_size]);  // 32 | group_size: one group
      uint32_t o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int lo = ((b[j] & 0xF) ^ 8) - 8, hi = ((b[j] >> 4) ^ 8) - 8;
        const __nv_bfloat162 bb = __floats2bfloat162_rn(static_cast<float>(lo) * s, static_cast<float>(hi) * s);
        o[j] = *reinterpret_cast<const uint32_t*>(&bb);
      }
      uint4* dst = reinterpret_cast<uint4*>(out + r * k + k0);
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
    }
  }
}

int dequant_to_bf16(int wfmt, const void* q, const void* scales, int group_size, int64_t rows, int64_t k, void* out,
                    cudaStream_t st) {
  if ((wfmt != SB_W_FP8 && wfmt != SB_W_INT4) || !q || !out || rows <= 0 || k % 64 ||
      (wfmt == SB_W_INT4 && (!scales || group_size <= 0 || group_size % 32 || k % group_size)) ||
      reinterpret_cast<uintptr_t>(q) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return SB_ERR_ARG;
  const int64_t chunks = rows * ((wfmt == SB_W_FP8 ? k : k / 2) / 16);
  int64_t blocks = (chunks + 255) / 256;
  const int64_t cap = 8 * current_sm_count();
  blocks = blocks > cap ? cap : blocks;
  return launch(dequant_bf16_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st,
                static_cast<const uint8_t*>(q), wfmt, static_cast<const __nv_bfloat16*>(scales), group_size, rows, k,
                static_cast<__nv_bfloat16*>(out));
}

int gemm_tcgen05(const sb_grouped_gemm_args& a, cudaStream_t st) {
  if (tc_qdec(a)) {
    const int rc = a.wfmt == SB_W_FP8 ? launch_qdec_epi<SB_W_FP8>(a, st) : launch_qdec_epi<SB_W_INT4>(a, st);
    if (rc != SB_ERR_UNSUPPORTED) return rc;
  }
  const int bn = tc_tile_n(a);
  switch (a.wfmt) {
    case SB_W_BF16: return launch_epi<SB_W_BF16>(a, st, bn);
    case SB_W_FP8: return launch_epi<SB_W_FP8>(a, st, bn);
    case SB_W_INT4: return launch_epi<SB_W_INT4>(a, st, bn);
    default: return SB_ERR_UNSUPPORTED;
  }
}

}  // namespace sb
