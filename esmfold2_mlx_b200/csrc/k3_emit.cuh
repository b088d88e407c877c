// K3: channel LayerNorm of the contraction output, output projection, output gate and the
// residual add, in one pass over the pair grid.
//
// Reference (src/esmfold2_mlx/): mlx_trunk.py:89-90,94-95; mlx_trunk_kernels.py:221-227 and the
// Metal kernels trunk_ln_cf_to_cl (:107-147) and trunk_resgate_ln (:165-190):
//   m     = fp16(LN_mix(x^T; norm_mix, mix_eps))     x is channel-major [B*c, L, Lpad]
//   mixed = fp16(m @ w_emit [+ b_emit])
//   g     = fp16(n @ w_out_gate [+ b_gate])            n = fp16(LN(z; norm_start)), as in K1
//   z'    = fp16(z + mixed * sigmoid(g))               fp32 math, one rounding
// The gate projection is recomputed here from the z tile this kernel must read anyway for the
// residual, instead of being written by K1 and read back: 512 fewer HBM bytes per pair cell.
// The LayerNorm that the reference fuses after the residual (resgate_ln's second output) is
// the next kernel's prologue (K1 of the next tri-mul normalises the z' it loads).
//
// One tile = 128 positions (ih x jw block).  CTA = 10 warps, one per SM, persistent:
//   warp 0     TMA: w_emit and w_gate once (resident), then per tile the z tile (2 stages,
//              128B swizzle, position-major) and the x tile (channel-major, unswizzled)
//   warp 1     TMEM (2 x 256 columns) + MMA thread: emit (A1 x W_e) and gate (A2 x W_g)
//   warps 2-5  transforms: A1 = fp16(LN_mix(x column)), A2 = fp16(LN_in(z row)), both written
//              as K-major 128B-swizzled UMMA operands
//   warps 6-9  epilogue: TMEM -> gate/residual in fp32 -> z' written over the z tile -> TMA store
#pragma once

#include "tmu_common.cuh"

namespace tmu {
namespace k3 {

constexpr int CZ = 128;
constexpr int CC = 128;
constexpr int TILE = 128;
constexpr int ATOM_BYTES = TILE * 128;
constexpr int TILE_BYTES = TILE * 128 * 2;  // 128 positions x 128 channels fp16
constexpr int OFF_WE = 0;
constexpr int OFF_WG = OFF_WE + CZ * CC * 2;
constexpr int OFF_Z = OFF_WG + CZ * CZ * 2;
constexpr int OFF_X = OFF_Z + 2 * TILE_BYTES;
constexpr int OFF_A1 = OFF_X + TILE * CC * 2;
constexpr int OFF_A2 = OFF_A1 + TILE_BYTES;
constexpr int SMEM_BYTES = OFF_A2 + TILE_BYTES + 1024;
constexpr int kThreads = 320;
constexpr int TMEM_COLS = 512;

struct Params {
  CUtensorMap tm_z;   // z [B, L, L, c_z]: box {64, jw, ih, 1}, 128B swizzle (load)
  CUtensorMap tm_zo;  // z_out, same geometry (store)
  CUtensorMap tm_x;   // x [B*c, L, Lpad]: box {jw, ih, c}, no swizzle (load)
  CUtensorMap tm_we;  // w_emit [c_z, c]: box {64, 128}
  CUtensorMap tm_wg;  // w_gate [c_z, c_z]: box {64, 128}
  const __half* ln_in_w;
  const __half* ln_in_b;
  const __half* ln_mix_w;
  const __half* ln_mix_b;
  const float* b_emit;  // [c_z] or null
  const float* b_gate;  // [c_z] or null
  float mix_eps;
  int L, ih, jw, tiles_i, tiles_j, num_tiles;
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProdZ = 0x301, kSiteProdX = 0x302, kSiteTrA = 0x303, kSiteTrX = 0x304, kSiteTrZ = 0x305,
  kSiteMmaW = 0x306, kSiteMmaA = 0x307, kSiteMmaT = 0x308, kSiteEpilogue = 0x309
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int per_b = p.tiles_i * p.tiles_j;
  bb = tile / per_b;
  const int r = tile - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

// LayerNorm of 128 fp16 values held as 16 uint4, written as fp16 to a K-major SW128 row.
__device__ __forceinline__ void ln_row_store(uint4 (&v)[16], const __half* w, const __half* b, float eps,
                                             uint8_t* dst, int row) {
  float sum = 0.f;
#pragma unroll
  for (int c16 = 0; c16 < 16; ++c16) {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[c16]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_half2(u[e]);
      sum += f.x + f.y;
    }
  }
  const float mean = sum * (1.0f / 128);
  float sq = 0.f;
#pragma unroll
  for (int c16 = 0; c16 < 16; ++c16) {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[c16]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_half2(u[e]);
      const float d0 = f.x - mean, d1 = f.y - mean;
      sq += d0 * d0 + d1 * d1;
    }
  }
  const float rstd = rsqrtf(sq * (1.0f / 128) + eps);
  const __half2* lw = reinterpret_cast<const __half2*>(w);
  const __half2* lb = reinterpret_cast<const __half2*>(b);
#pragma unroll
  for (int c16 = 0; c16 < 16; ++c16) {
    uint32_t* u = reinterpret_cast<uint32_t*>(&v[c16]);
    uint4 o;
    uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_half2(u[e]);
      const float2 g = __half22float2(__ldg(lw + c16 * 4 + e));
      const float2 bb = __half22float2(__ldg(lb + c16 * 4 + e));
      ou[e] = pack_half2((f.x - mean) * rstd * g.x + bb.x, (f.y - mean) * rstd * g.y + bb.y);
    }
    *reinterpret_cast<uint4*>(dst + (c16 >> 3) * ATOM_BYTES + sw128_off(row, c16 & 7)) = o;
  }
}

__global__ void __launch_bounds__(kThreads, 1) emit_residual_kernel(const __grid_constant__ Params p) {
  constexpr uint32_t IDESC = idesc_f16_f32(128, CZ, false, false);
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t w_bar, zfull[2], zempty[2], xfull, xempty, afull, aempty;
  __shared__ __align__(8) uint64_t tfull[2], tempty[2], drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  __shared__ volatile int ep_ok_sh;

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&w_bar, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&zfull[s], 1);
      mbar_init(&zempty[s], 1);
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 128);
    }
    mbar_init(&xfull, 1);
    mbar_init(&xempty, 128);
    mbar_init(&afull, 128);
    mbar_init(&aempty, 1);
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_z);
    tma_prefetch_desc(&p.tm_zo);
    tma_prefetch_desc(&p.tm_x);
    tma_prefetch_desc(&p.tm_we);
    tma_prefetch_desc(&p.tm_wg);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(&w_bar, (CZ * CC + CZ * CZ) * 2);
      for (int a = 0; a < CC / 64; ++a) tma_load_2d(smem + OFF_WE + a * ATOM_BYTES, &p.tm_we, &w_bar, a * 64, 0);
      for (int a = 0; a < CZ / 64; ++a) tma_load_2d(smem + OFF_WG + a * ATOM_BYTES, &p.tm_wg, &w_bar, a * 64, 0);
      uint32_t it = 0, nz = 0, nx = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        if (!mbar_wait(&zempty[s], ph ^ 1, ctx, kSiteProdZ)) break;
        mbar_arrive_expect_tx(&zfull[s], TILE_BYTES);
        for (int a = 0; a < CZ / 64; ++a)
          tma_load_4d(smem + OFF_Z + s * TILE_BYTES + a * ATOM_BYTES, &p.tm_z, &zfull[s], a * 64, j0, i0, bb);
        ++nz;
        if (!mbar_wait(&xempty, (it & 1) ^ 1, ctx, kSiteProdX)) break;
        mbar_arrive_expect_tx(&xfull, TILE * CC * 2);
        tma_load_3d(smem + OFF_X, &p.tm_x, &xfull, j0, i0, bb * CC);
        ++nx;
      }
      if (abort_sh) {
        mbar_drain(&w_bar, 0, 200000000ull);
        for (uint32_t s = 0; s < 2; ++s) {
          const uint32_t n_armed = nz > s ? (nz - s + 1) / 2 : 0;
          if (n_armed) mbar_drain(&zfull[s], (n_armed - 1) & 1, 200000000ull);
        }
        if (nx) mbar_drain(&xfull, (nx - 1) & 1, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = mbar_wait(&w_bar, 0, ctx, kSiteMmaW);
      uint32_t it = 0;
      const uint32_t a1 = smem_u32(smem + OFF_A1), a2 = smem_u32(smem + OFF_A2);
      const uint32_t we = smem_u32(smem + OFF_WE), wg = smem_u32(smem + OFF_WG);
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
        const uint32_t acc = it & 1, aph = (it >> 1) & 1;
        if (!mbar_wait(&afull, it & 1, ctx, kSiteMmaA)) break;
        if (!mbar_wait(&tempty[acc], aph ^ 1, ctx, kSiteMmaT)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * 256;
#pragma unroll
        for (int kk = 0; kk < CC / 16; ++kk) {
          const uint32_t off = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
          umma_f16(d, sdesc_sw128(a1 + off, 16, 1024), sdesc_sw128(we + off, 16, 1024), IDESC, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < CZ / 16; ++kk) {
          const uint32_t off = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
          umma_f16(d + CZ, sdesc_sw128(a2 + off, 16, 1024), sdesc_sw128(wg + off, 16, 1024), IDESC,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(&aempty);
        umma_commit(&tfull[acc]);
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < 6) {
    // ---------------- operand transforms ----------------
    const int row = threadIdx.x - 64;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const uint32_t s = it & 1, ph = (it >> 1) & 1;
      if (!mbar_wait(&aempty, (it & 1) ^ 1, ctx, kSiteTrA)) break;
      if (!mbar_wait(&xfull, it & 1, ctx, kSiteTrX)) break;
      {
        // x tile is [channel][position]: gather this position's column
        const __half* X = reinterpret_cast<const __half*>(smem + OFF_X);
        uint4 v[16];
#pragma unroll
        for (int c16 = 0; c16 < 16; ++c16) {
          uint32_t* u = reinterpret_cast<uint32_t*>(&v[c16]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int ch = c16 * 8 + e * 2;
            __half2 h2 = __halves2half2(X[ch * TILE + row], X[(ch + 1) * TILE + row]);
            u[e] = *reinterpret_cast<uint32_t*>(&h2);
          }
        }
        mbar_arrive(&xempty);
        ln_row_store(v, p.ln_mix_w, p.ln_mix_b, p.mix_eps, smem + OFF_A1, row);
      }
      if (!mbar_wait(&zfull[s], ph, ctx, kSiteTrZ)) break;
      {
        const uint8_t* Z = smem + OFF_Z + s * TILE_BYTES;
        uint4 v[16];
#pragma unroll
        for (int c16 = 0; c16 < 16; ++c16)
          v[c16] = *reinterpret_cast<const uint4*>(Z + (c16 >> 3) * ATOM_BYTES + sw128_off(row, c16 & 7));
        ln_row_store(v, p.ln_in_w, p.ln_in_b, 1e-5f, smem + OFF_A2, row);
      }
      fence_proxy_async_smem();
      mbar_arrive(&afull);
    }
  } else {
    // ---------------- epilogue ----------------
    const int e = threadIdx.x - 192;  // 0..127
    const int q = warp & 3;
    const int row = q * 32 + lane;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t s = it & 1, ph = (it >> 1) & 1;
      const uint32_t acc = it & 1, aph = (it >> 1) & 1;
      if (e == 0) {
        ep_ok_sh = (mbar_wait(&tfull[acc], aph, ctx, kSiteEpilogue) && mbar_wait(&zfull[s], ph, ctx, kSiteEpilogue))
                       ? 1 : 0;
      }
      named_bar_sync(2, 128);
      if (!ep_ok_sh) break;
      tc_fence_after();
      uint8_t* Z = smem + OFF_Z + s * TILE_BYTES;
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * 256;
#pragma unroll 1
      for (int cc = 0; cc < CZ / 32; ++cc) {
        uint32_t em[32], gt[32];
        tmem_ld32(trow + cc * 32, em);
        tmem_ld32(trow + CZ + cc * 32, gt);
        tmem_wait_ld2(em, gt);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c16 = (cc & 1) * 4 + j;
          uint8_t* zp = Z + (cc >> 1) * ATOM_BYTES + sw128_off(row, c16);
          uint4 zv = *reinterpret_cast<const uint4*>(zp);
          uint32_t* zu = reinterpret_cast<uint32_t*>(&zv);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int i = j * 8 + k * 2;
            const int n = cc * 32 + i;
            float m0 = __uint_as_float(em[i]), m1 = __uint_as_float(em[i + 1]);
            float g0 = __uint_as_float(gt[i]), g1 = __uint_as_float(gt[i + 1]);
            if (p.b_emit != nullptr) {
              m0 += __ldg(p.b_emit + n);
              m1 += __ldg(p.b_emit + n + 1);
            }
            if (p.b_gate != nullptr) {
              g0 += __ldg(p.b_gate + n);
              g1 += __ldg(p.b_gate + n + 1);
            }
            m0 = round_f16(m0);
            m1 = round_f16(m1);
            g0 = round_f16(g0);
            g1 = round_f16(g1);
            const float2 zf = unpack_half2(zu[k]);
            zu[k] = pack_half2(zf.x + m0 * sigmoid_f32(g0), zf.y + m1 * sigmoid_f32(g1));
          }
          *reinterpret_cast<uint4*>(zp) = zv;
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      fence_proxy_async_smem();
      named_bar_sync(2, 128);
      if (e == 0) {
        for (int a = 0; a < CZ / 64; ++a) tma_store_4d(&p.tm_zo, Z + a * ATOM_BYTES, a * 64, j0, i0, bb);
        bulk_commit();
        bulk_wait_read<0>();
        mbar_arrive(&zempty[s]);
      }
    }
    if (e == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace k3
}  // namespace tmu
