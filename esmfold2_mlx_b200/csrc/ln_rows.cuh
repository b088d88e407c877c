// LayerNorm of pair-grid rows read straight from global memory by one warp per row, written as
// fp16 into a K-major 128B-swizzled MMA operand tile (atoms of 128 rows x 64 channels).
//
// Lane l holds channels 4(l + 32q) .. 4(l + 32q) + 3 for q < NQ = K / 128, so every load
// instruction of the warp reads 32 x 16 B (fp32) or 32 x 8 B (fp16) contiguous bytes of the row.
// Plain (coherent) loads: a kernel may write the rows it normalised later in the same launch.
// Statistics are fp32 and two-pass over the registers: mean = sum(x) / K, then
// var = sum((x - mean)^2) / K, each a warp all-reduce; y = (x - mean) * rstd * gamma + beta, rounded
// once to fp16 (gamma/beta absent: y = (x - mean) * rstd).
#pragma once

#include "tmu_common.cuh"

namespace tmu {

__device__ __forceinline__ float warp_allsum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Where a row comes from: one fp32 or fp16 tensor, the concatenation of two fp32 tensors of K/2
// channels each (channels [0, K/2) from x1, [K/2, K) from x2), or the sum of two fp32 tensors.
enum RowSrc : int { kRowF32 = 0, kRowF16 = 1, kRowCat32 = 2, kRowSum32 = 3 };

template <int SRC, int NQ>
__device__ __forceinline__ void load_row(const void* x1, const void* x2, size_t cell, int ld1, int ld2, int lane,
                                         float4 (&v)[NQ]) {
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    if constexpr (SRC == kRowF32) {
      v[q] = reinterpret_cast<const float4*>(static_cast<const float*>(x1) + cell * ld1)[lane + 32 * q];
    } else if constexpr (SRC == kRowF16) {
      const uint2 u = reinterpret_cast<const uint2*>(static_cast<const __half*>(x1) + cell * ld1)[lane + 32 * q];
      const float2 a = unpack_half2(u.x), b = unpack_half2(u.y);
      v[q] = make_float4(a.x, a.y, b.x, b.y);
    } else if constexpr (SRC == kRowCat32) {
      const float* base = q < NQ / 2 ? static_cast<const float*>(x1) + cell * ld1
                                     : static_cast<const float*>(x2) + cell * ld2;
      v[q] = __ldg(reinterpret_cast<const float4*>(base) + lane + 32 * (q % (NQ / 2)));
    } else {  // kRowSum32
      const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(x1) + cell * ld1) + lane + 32 * q);
      const float4 b = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(x2) + cell * ld2) + lane + 32 * q);
      v[q] = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
    }
  }
}

// gamma/beta of this lane's channels (or identity when g == nullptr)
template <int NQ>
__device__ __forceinline__ void load_ln_par(const float* g, const float* b, int lane, float4 (&gg)[NQ],
                                            float4 (&bb)[NQ]) {
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    gg[q] = g ? __ldg(reinterpret_cast<const float4*>(g) + lane + 32 * q) : make_float4(1.f, 1.f, 1.f, 1.f);
    bb[q] = b ? __ldg(reinterpret_cast<const float4*>(b) + lane + 32 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Normalise the row held in v and write it to row `row` of the swizzled tile at `tile`.
// affine == false skips gamma/beta (mx.fast.layer_norm(x, None, None, eps)).
template <int NQ>
__device__ __forceinline__ void ln_row_store(const float4 (&v)[NQ], const float4 (&gg)[NQ], const float4 (&bb)[NQ],
                                             bool affine, float eps, uint8_t* tile, int atom_bytes, int row,
                                             int lane) {
  constexpr float inv_k = 1.0f / (128 * NQ);
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < NQ; ++q) s += (v[q].x + v[q].y) + (v[q].z + v[q].w);
  const float mean = warp_allsum(s) * inv_k;
  float s2 = 0.f;
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const float a = v[q].x - mean, b = v[q].y - mean, c = v[q].z - mean, d = v[q].w - mean;
    s2 = fmaf(a, a, s2);
    s2 = fmaf(b, b, s2);
    s2 = fmaf(c, c, s2);
    s2 = fmaf(d, d, s2);
  }
  const float rstd = rsqrtf(warp_allsum(s2) * inv_k + eps);
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    float2 lo = make_float2((v[q].x - mean) * rstd, (v[q].y - mean) * rstd);
    float2 hi = make_float2((v[q].z - mean) * rstd, (v[q].w - mean) * rstd);
    if (affine) {
      lo = make_float2(fmaf(lo.x, gg[q].x, bb[q].x), fmaf(lo.y, gg[q].y, bb[q].y));
      hi = make_float2(fmaf(hi.x, gg[q].z, bb[q].z), fmaf(hi.y, gg[q].w, bb[q].w));
    }
    const int c0 = 4 * (lane + 32 * q);  // first channel of this lane's four
    uint8_t* dst = tile + (c0 >> 6) * atom_bytes + sw128_off(row, (c0 & 63) >> 3) + (c0 & 4) * 2;
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_half2(lo.x, lo.y), pack_half2(hi.x, hi.y));
  }
}

// A row past the grid's edge (a tile overhanging L): zeros, so the MMA reads defined values.
template <int NQ>
__device__ __forceinline__ void zero_row_store(uint8_t* tile, int atom_bytes, int row, int lane) {
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int c0 = 4 * (lane + 32 * q);
    uint8_t* dst = tile + (c0 >> 6) * atom_bytes + sw128_off(row, (c0 & 63) >> 3) + (c0 & 4) * 2;
    *reinterpret_cast<uint2*>(dst) = make_uint2(0u, 0u);
  }
}

}  // namespace tmu
