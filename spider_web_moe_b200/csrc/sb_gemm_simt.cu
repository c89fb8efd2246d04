// CUDA-core grouped GEMM: the fp32 engine (the reference block's own precision,
// used for fp32 workloads) and the independent cross-check of the tcgen05
// engine.  Same operands, schedule and epilogues as sb_gemm_tc.cu.
#include "sb_gemm_common.cuh"
#include "sb_internal.h"

namespace sb {

constexpr int kSimtBM = 64, kSimtBN = 32, kSimtBK = 32, kSimtThreads = 256;

struct SimtParams {
  sb_grouped_gemm_args a;
};

// Load A[row, k] of any weight format as fp32 (fp8: raw e4m3 value, the row
// scale is applied in the epilogue; int4: dequantised and rounded to bf16).
SB_DEVINL float load_weight(const sb_grouped_gemm_args& p, const void* base, const void* scale,
                            int64_t row, int k) {
  switch (p.wfmt) {
    case SB_W_F32:
      return static_cast<const float*>(base)[row * p.lda + k];
    case SB_W_BF16:
      return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[row * p.lda + k]);
    case SB_W_FP8:
      return fp8e4m3_to_f32(static_cast<const uint8_t*>(base)[row * p.lda + k]);
    default: {
      const uint8_t b = static_cast<const uint8_t*>(base)[row * (p.lda / 2) + (k >> 1)];
      const int groups = static_cast<int>(p.lda / p.group_size);
      const float s = __bfloat162float(
          static_cast<const __nv_bfloat16*>(scale)[row * groups + k / p.group_size]);
      return int4_weight(b, k & 1, s);
    }
  }
}

// fp8 weights, or bf16 weights with a per-row scale (fp8 weights converted exactly)
SB_DEVINL float row_scale_of(const sb_grouped_gemm_args& p, const void* scale, int64_t row) {
  return (p.wfmt == SB_W_FP8 || (p.wfmt == SB_W_BF16 && scale)) ? static_cast<const float*>(scale)[row] : 1.f;
}

// kIL: interleaved SwiGLU (SB_EPI_SWIGLU_IL) -- a CTA's 64 output features
// have their gate rows at 128 * (m0 / 64) .. + 63 of the group and their up
// rows 64 further; both come from `a`.
template <bool kGate, bool kIL = false>
__global__ void __launch_bounds__(kSimtThreads)
simt_gemm_kernel(const sb_grouped_gemm_args p) {
  __shared__ float As[kSimtBK][kSimtBM + 4];
  __shared__ float Gs[kGate ? kSimtBK : 1][kSimtBM + 4];
  __shared__ float Bs[kSimtBK][kSimtBN + 4];
  __shared__ int s_sched[4];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x;
  if (tid < 32) {
    int g, n0, n_end;
    const bool ok = schedule_tile(p.offsets, p.num_groups, kSimtBN, blockIdx.y, g, n0, n_end, p.max_rows);
    if (tid == 0) {
      s_sched[0] = ok ? g : -1;
      s_sched[1] = n0;
      s_sched[2] = min(n_end, p.max_rows);
    }
  }
  __syncthreads();
  const int g = s_sched[0];
  if (g < 0) return;
  const int n0 = s_sched[1], n_end = s_sched[2];
  const int m0 = blockIdx.x * kSimtBM;
  const int ks = p.k / p.splits;
  const int kb = blockIdx.z * ks, ke = (blockIdx.z == p.splits - 1) ? p.k : kb + ks;
  const int m_out = kIL ? p.m_rows / 2 : p.m_rows;   // output features
  const int lrow0 = kIL ? 2 * m0 + 64 : m0;          // group-local row of feature m0 (the up row)
  const int64_t arow0 = static_cast<int64_t>(g) * p.a_group_rows + lrow0;
  const int64_t grow0 = kIL ? arow0 - 64 : arow0;    // its gate row (interleaved layout)
  const void* gate_w = kIL ? p.a : p.a_gate;
  const void* gate_s = kIL ? p.a_scale : p.a_gate_scale;

  const int tx = tid % 16, ty = tid / 16;  // rows n = 2*tx + j, features m = 4*ty + i
  float acc[4][2] = {}, accg[4][2] = {};
  for (int k0 = kb; k0 < ke; k0 += kSimtBK) {
    for (int i = tid; i < kSimtBM * kSimtBK; i += kSimtThreads) {
      const int mm = i / kSimtBK, kk = i % kSimtBK;
      const int64_t row = arow0 + mm;
      const bool ok = (m0 + mm) < m_out && row < p.a_rows_total && (k0 + kk) < ke;
      As[kk][mm] = ok ? load_weight(p, p.a, p.a_scale, row, k0 + kk) : 0.f;
      if (kGate) Gs[kk][mm] = ok ? load_weight(p, gate_w, gate_s, grow0 + mm, k0 + kk) : 0.f;
    }
    for (int i = tid; i < kSimtBN * kSimtBK; i += kSimtThreads) {
      const int nn = i / kSimtBK, kk = i % kSimtBK;
      const int r = n0 + nn;
      float v = 0.f;
      if (r < n_end && (k0 + kk) < ke) {
        const int64_t src_row = p.x_row_index ? p.x_row_index[r] : r;
        const int64_t off = src_row * p.ldx + k0 + kk;
        v = p.act_dtype == SB_F32 ? static_cast<const float*>(p.x)[off]
                                  : __bfloat162float(static_cast<const __nv_bfloat16*>(p.x)[off]);
      }
      Bs[kk][nn] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kSimtBK; ++kk) {
      float bv[2] = {Bs[kk][2 * tx], Bs[kk][2 * tx + 1]};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float av = As[kk][4 * ty + i];
        acc[i][0] = fmaf(av, bv[0], acc[i][0]);
        acc[i][1] = fmaf(av, bv[1], acc[i][1]);
        if (kGate) {
          const float gv = Gs[kk][4 * ty + i];
          accg[i][0] = fmaf(gv, bv[0], accg[i][0]);
          accg[i][1] = fmaf(gv, bv[1], accg[i][1]);
        }
      }
    }
    __syncthreads();
  }
  // epilogue
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + 4 * ty + i;
    if (m >= m_out) continue;
    const int64_t row = arow0 + 4 * ty + i;
    const int lrow = lrow0 + 4 * ty + i;  // group-local weight row (bias index)
    const float sa = row_scale_of(p, p.a_scale, row);
    const float bias = (p.bias && blockIdx.z == 0) ? p.bias[static_cast<int64_t>(g) * p.bias_group_stride + lrow] : 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int r = n0 + 2 * tx + j;
      if (r >= n_end) continue;
      const float v = acc[i][j] * sa + bias;
      if (p.epilogue == SB_EPI_LINEAR) {
        const float rs = p.row_scale ? p.row_scale[r] : 1.f;
        static_cast<float*>(p.out)[blockIdx.z * p.split_stride + static_cast<int64_t>(r) * p.ldo + m] = v * rs;
      } else {
        float o;
        if (p.epilogue == SB_EPI_GELU) {
          o = gelu_erf(v);
        } else {
          const float sg = row_scale_of(p, gate_s, grow0 + 4 * ty + i);
          const float* gb = kIL ? p.bias : p.bias_gate;
          const float bg = gb ? gb[static_cast<int64_t>(g) * p.bias_group_stride + (kIL ? lrow - 64 : m)] : 0.f;
          o = silu(accg[i][j] * sg + bg) * v;
        }
        if (p.act_dtype == SB_F32)
          static_cast<float*>(p.out)[static_cast<int64_t>(r) * p.ldo + m] = o;
        else
          static_cast<__nv_bfloat16*>(p.out)[static_cast<int64_t>(r) * p.ldo + m] = __float2bfloat16_rn(o);
      }
    }
  }
}

int gemm_simt(const sb_grouped_gemm_args& a, cudaStream_t st) {
  const bool il = a.epilogue == SB_EPI_SWIGLU_IL;
  if (il && a.m_rows % 128) return SB_ERR_UNSUPPORTED;
  const int m_tiles = ((il ? a.m_rows / 2 : a.m_rows) + kSimtBM - 1) / kSimtBM;
  const int n_slots = (a.max_rows + kSimtBN - 1) / kSimtBN + a.num_groups;
  const dim3 grid(m_tiles, n_slots, a.splits);
  if (il) return launch(simt_gemm_kernel<true, true>, grid, dim3(kSimtThreads), 0, st, a);
  if (a.epilogue == SB_EPI_SWIGLU) return launch(simt_gemm_kernel<true>, grid, dim3(kSimtThreads), 0, st, a);
  return launch(simt_gemm_kernel<false>, grid, dim3(kSimtThreads), 0, st, a);
}

}  // namespace sb
