// Row LayerNorm pass over the pair grid: h[row] = fp16(LN(x[row])), written row-major for a TMA
// tile map over [B, L, L, K] to read.  The GEMM kernels of the diffusion pair conditioning
// (K6, K4 in h mode) take their A operand from it.
//
// One warp per row: lane l holds channels 4(l + 32q) .. 4(l + 32q) + 3 for q < NQ = K / 128, so
// every load instruction of the warp reads 32 x 16 B (fp32) or 32 x 8 B (fp16) contiguous bytes.
// Statistics are fp32 and two-pass over the registers: mean = sum(x) / K, then
// var = sum((x - mean)^2) / K, each a warp all-reduce; y = (x - mean) * rstd * gamma + beta, rounded
// once to fp16 (gamma/beta absent: y = (x - mean) * rstd).
#pragma once

#include <cuda_bf16.h>

#include "tmu_common.cuh"

namespace tmu {

__device__ __forceinline__ float warp_allsum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Where a row comes from: one fp32 or fp16 tensor, the concatenation of two fp32 tensors of K/2
// channels each (channels [0, K/2) from x1, [K/2, K) from x2), the sum of two fp32 tensors, or
// an fp32 sum of fp16 terms (RowTerms below).
enum RowSrc : int { kRowF32 = 0, kRowF16 = 1, kRowCat32 = 2, kRowSum32 = 3, kRowTerms16 = 4 };

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

// A row held as an fp32 sum of fp16 terms, z = fl32(fl32(s0 + s1) + s2) ..., added in source
// order: a residual stream kept as its fp16 increments (z0 and each transition's rounded output)
// gives back exactly the fp32 value a running fp32 sum would hold.
constexpr int kMaxTerms = 4;

struct RowTerms {
  const __half* src[kMaxTerms];
  int n;   // 1 .. kMaxTerms
  int ld;  // row pitch, elements (the same for every term)
};

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

namespace lnr {

// h[row] = fp16(LN(x[row])) for `rows` rows of K channels.  RL rows in flight per warp and many
// warps per SM, so the loads of this memory-bound pass overlap.
constexpr int kThreads = 256;

struct Params {
  const void* x1;
  const void* x2;
  int ld1, ld2;
  RowTerms terms;
  const float* g;  // [K] or null
  const float* b;
  void* out;       // kOutF16: fp16 [rows, K]; kOutBf16x3: bf16 [rows, 3K]
  long long rows;
  float eps;
};

// kOutF16:    h = fp16(y), one rounding.
// kOutBf16x3: y split exactly into three bf16 parts, y = y0 + y1 + y2 to 24 significant bits
//             (y0 = bf16(y), y1 = bf16(y - y0), y2 = bf16(y - y0 - y1)), stored as channel blocks
//             [y0 | y1 | y2] of a 3K-wide row: the A operand of an fp32-accurate tensor-core GEMM.
enum Out : int { kOutF16 = 0, kOutBf16x3 = 1 };

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t u) {
  const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

template <int K, int SRC, int OUT = kOutF16>
__global__ void __launch_bounds__(kThreads) ln_rows_kernel(const __grid_constant__ Params p) {
  constexpr int NQ = K / 128;
  constexpr int RL = K <= 256 ? 4 : 2;
  // fp16 terms: every load of the RL rows (all terms, kMaxTerms of them predicated by the count)
  // is issued before the first add, so the rows' memory latencies overlap.
  constexpr int NT = SRC == kRowTerms16 ? kMaxTerms : 1;
  const int lane = threadIdx.x & 31;
  const long long warp0 = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(gridDim.x) * kThreads) >> 5;
  float4 gg[NQ], bb[NQ];
  load_ln_par<NQ>(p.g, p.b, lane, gg, bb);
  const bool affine = p.g != nullptr;
  griddep_wait();  // the rows may be the previous kernel's output
  for (long long r0 = warp0 * RL; r0 < p.rows; r0 += nwarps * RL) {
    float4 v[RL][NQ];
    if constexpr (SRC == kRowTerms16) {
      uint2 raw[RL][NT][NQ];
#pragma unroll
      for (int u = 0; u < RL; ++u)
#pragma unroll
        for (int k = 0; k < NT; ++k)
#pragma unroll
          for (int q = 0; q < NQ; ++q)
            raw[u][k][q] = (r0 + u < p.rows && k < p.terms.n)
                               ? reinterpret_cast<const uint2*>(p.terms.src[k] + static_cast<size_t>(r0 + u) * p.terms.ld)[lane + 32 * q]
                               : make_uint2(0u, 0u);
#pragma unroll
      for (int u = 0; u < RL; ++u)
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
          float2 a = unpack_half2(raw[u][0][q].x), b = unpack_half2(raw[u][0][q].y);
          v[u][q] = make_float4(a.x, a.y, b.x, b.y);
#pragma unroll
          for (int k = 1; k < NT; ++k)
            if (k < p.terms.n) {  // fl32(fl32(t0 + t1) + t2) ..., in term order
              a = unpack_half2(raw[u][k][q].x);
              b = unpack_half2(raw[u][k][q].y);
              v[u][q] = make_float4(v[u][q].x + a.x, v[u][q].y + a.y, v[u][q].z + b.x, v[u][q].w + b.y);
            }
        }
    } else {
#pragma unroll
      for (int u = 0; u < RL; ++u)
        if (r0 + u < p.rows) load_row<SRC, NQ>(p.x1, p.x2, static_cast<size_t>(r0 + u), p.ld1, p.ld2, lane, v[u]);
    }
#pragma unroll
    for (int u = 0; u < RL; ++u) {
      const long long row = r0 + u;
      if (row >= p.rows) break;
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < NQ; ++q) s += (v[u][q].x + v[u][q].y) + (v[u][q].z + v[u][q].w);
      const float mean = warp_allsum(s) * (1.0f / K);
      float s2 = 0.f;
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const float a = v[u][q].x - mean, b = v[u][q].y - mean, c = v[u][q].z - mean, d = v[u][q].w - mean;
        s2 = fmaf(a, a, s2);
        s2 = fmaf(b, b, s2);
        s2 = fmaf(c, c, s2);
        s2 = fmaf(d, d, s2);
      }
      const float rstd = rsqrtf(warp_allsum(s2) * (1.0f / K) + p.eps);
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        float2 lo = make_float2((v[u][q].x - mean) * rstd, (v[u][q].y - mean) * rstd);
        float2 hi = make_float2((v[u][q].z - mean) * rstd, (v[u][q].w - mean) * rstd);
        if (affine) {
          lo = make_float2(fmaf(lo.x, gg[q].x, bb[q].x), fmaf(lo.y, gg[q].y, bb[q].y));
          hi = make_float2(fmaf(hi.x, gg[q].z, bb[q].z), fmaf(hi.y, gg[q].w, bb[q].w));
        }
        if constexpr (OUT == kOutF16) {
          uint2* dst = reinterpret_cast<uint2*>(static_cast<__half*>(p.out) + static_cast<size_t>(row) * K);
          dst[lane + 32 * q] = make_uint2(pack_half2(lo.x, lo.y), pack_half2(hi.x, hi.y));
        } else {
          uint2* dst = reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(row) * 3 * K);
          float y[4] = {lo.x, lo.y, hi.x, hi.y};
#pragma unroll
          for (int part = 0; part < 3; ++part) {
            const uint32_t w0 = pack_bf16x2(y[0], y[1]), w1 = pack_bf16x2(y[2], y[3]);
            dst[part * (K / 4) + lane + 32 * q] = make_uint2(w0, w1);
            const float2 r0 = unpack_bf16x2(w0), r1 = unpack_bf16x2(w1);
            y[0] -= r0.x;  // exact: the remainder of a bf16 rounding of an fp32 value
            y[1] -= r0.y;
            y[2] -= r1.x;
            y[3] -= r1.y;
          }
        }
      }
    }
  }
  griddep_trigger();
}

}  // namespace lnr
}  // namespace tmu
