// Pieces shared by the two grouped-GEMM engines.
#pragma once
#include "sb_common.cuh"

namespace sb {

// Device-side tile schedule.  Group g owns permuted rows [offsets[g],
// offsets[g+1]) and ceil(count/BN) column tiles; tiles are numbered group by
// group.  Executed by one full warp; returns false (uniformly) when `slot` is
// beyond the last tile.  No host synchronisation is needed: the launch grid is
// an upper bound and surplus CTAs leave at once.
// Row offset of group g; offsets == nullptr means one dense group of max_rows rows.
SB_DEVINL int group_offset(const int32_t* __restrict__ offsets, int g, int max_rows) {
  return offsets ? offsets[g] : (g == 0 ? 0 : max_rows);
}

SB_DEVINL bool schedule_tile(const int32_t* __restrict__ offsets, int G, int BN, int slot, int& g,
                             int& n0, int& n_end, int max_rows) {
  const int lane = threadIdx.x & 31;
  int seen = 0;
  int found_g = -1, found_n0 = 0, found_end = 0;
  for (int base = 0; base < G; base += 32) {
    const int gi = base + lane;
    int lo = 0, hi = 0;
    if (gi < G) {
      lo = group_offset(offsets, gi, max_rows);
      hi = group_offset(offsets, gi + 1, max_rows);
    }
    const int cnt = hi > lo ? hi - lo : 0;
    const int tiles = (cnt + BN - 1) / BN;
    int incl = tiles;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += t;
    }
    const int excl = seen + incl - tiles;
    const bool mine = gi < G && slot >= excl && slot < excl + tiles;
    const unsigned who = __ballot_sync(0xffffffffu, mine);
    if (who) {
      const int src = __ffs(who) - 1;
      found_g = __shfl_sync(0xffffffffu, gi, src);
      found_n0 = __shfl_sync(0xffffffffu, lo + (slot - excl) * BN, src);
      found_end = __shfl_sync(0xffffffffu, hi, src);
      break;
    }
    seen += __shfl_sync(0xffffffffu, incl, 31);
  }
  g = found_g;
  n0 = found_n0;
  n_end = found_end;
  return found_g >= 0;
}

// e4m3 byte -> float (exact).
SB_DEVINL float fp8e4m3_to_f32(uint8_t b) {
  __nv_fp8_e4m3 v;
  v.__x = b;
  return static_cast<float>(v);
}

// Signed nibble of a packed int4 byte (even element in the low nibble).
SB_DEVINL int int4_nibble(uint8_t b, int hi) {
  const int v = hi ? (b >> 4) : (b & 0xF);
  return (v ^ 8) - 8;
}

// Dequantised int4 weight as the bf16 value both engines multiply with.
SB_DEVINL float int4_weight(uint8_t b, int hi, float scale) {
  return __bfloat162float(__float2bfloat16_rn(static_cast<float>(int4_nibble(b, hi)) * scale));
}

}  // namespace sb
