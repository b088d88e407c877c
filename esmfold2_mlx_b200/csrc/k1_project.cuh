// K1: input LayerNorm + the four c_z -> c projections of the contraction operands, sigmoid
// gating and the pair mask, written channel-major for the contraction (no transpose pass).
//
// Reference (src/esmfold2_mlx/): mlx_trunk.py:81-83 and :72-76 (_gated_cf);
// mlx_trunk_kernels.py:214-216 and the Metal kernel trunk_gate_cf (:47-80):
//   n     = fp16(LN(z; norm_start, eps=1e-5))                    fp32 statistics
//   proj  = fp16(n @ w_in [+ b_in])                                fp32 accumulation
//   a     = fp16(proj[:, 0:c]  * sigmoid(proj[:, 2c:3c]) * mask)   fp32 math, one rounding
//   b     = fp16(proj[:, c:2c] * sigmoid(proj[:, 3c:4c]) * mask)
// a, b stored [B*c, L, Lpad] (channel d, row i, column j).  The fp16 pre-scale of w_in[:, :c]
// by 1/256 (mlx_trunk.py:47-48) lives in the packed weights.
//
// One tile = 128 pair positions, an ih x jw block of the L x L grid (ih * jw = 128), chosen by
// the host to minimise padding at ragged L.  CTA = 18 warps, one per SM, persistent:
//   warp 0      TMA: packed weights once (resident, 4c x c_z fp16), then z tiles (2 stages)
//   warp 1      TMEM allocation (512 columns = 4 slots of 128) and the single MMA thread:
//               per tile, NCH chunks of N = 128 columns ([signal 64 | gate 64] of one 64-channel
//               block of a or b), K = c_z, each chunk into the next TMEM slot
//   warps 2-5   LayerNorm of the z tile in shared memory, in place (thread = position)
//   warps 6-17  epilogue, three groups of four warps (one per TMEM lane quadrant); group g takes
//               the chunks with (chunk index % 3 == g), so three chunks drain at once.  Each warp
//               owns 32 positions: gate, mask, fp16, then a 16-channel x 32-position block is
//               staged in shared memory and stored with its own TMA store (no CTA-wide barrier).
#pragma once

#include "tmu_common.cuh"

namespace tmu {
namespace k1 {

constexpr int CZ = 128;  // c_z
constexpr int CC = 128;  // c (latent channels)
constexpr int TILE = 128;
constexpr int NCH = 4 * CC / 128;       // 128-column chunks per tile
constexpr int KATOMS = CZ / 64;         // 64-channel swizzle atoms along K
constexpr int ATOM_BYTES = TILE * 128;  // 128 rows x 128 B
constexpr int WCHUNK_BYTES = 128 * CZ * 2;
constexpr int A_BYTES = TILE * CZ * 2;
constexpr int NSTAGE = 2;
constexpr int NSLOT = 4;
constexpr int SUB = 16;                      // channels per epilogue store
constexpr int WSTG_BYTES = SUB * 32 * 2;     // one warp's staging buffer (16 ch x 32 positions)
constexpr int OFF_W = 0;
constexpr int OFF_A = OFF_W + NCH * WCHUNK_BYTES;
constexpr int OFF_STG = OFF_A + NSTAGE * A_BYTES;
constexpr int NEPI = 12;                                 // epilogue warps (3 groups of 4)
constexpr int OFF_PAR = OFF_STG + NEPI * 2 * WSTG_BYTES;  // fp32 LN gamma, beta, bias
constexpr int PAR_FLOATS = 2 * CZ + 4 * CC;
constexpr int SMEM_BYTES = OFF_PAR + PAR_FLOATS * 4 + 1024;
constexpr int kThreads = 576;
constexpr int TMEM_COLS = 512;

struct Params {
  CUtensorMap tm_z;  // z [B, L, L, c_z]: box {64, jw, ih, 1}, 128B swizzle
  CUtensorMap tm_w;  // packed proj weights [4c, c_z]: box {64, 128}, 128B swizzle
  CUtensorMap tm_a;  // a [B*c, L, Lpad]: box {min(jw,32), 32/min(jw,32), 16}, no swizzle (store)
  CUtensorMap tm_b;  // b, same
  const __half* ln_w;
  const __half* ln_b;
  const float* bias;   // [4c] in packed-row order, or null
  const __half* mask;  // [B, L, L] or null
  int L, ih, jw, tiles_i, tiles_j, num_tiles;
  int reset_status;  // block 0 zeroes the status word (after the dependency wait)
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProducer = 0x101, kSiteLn = 0x102, kSiteMmaW = 0x103, kSiteMmaLn = 0x104, kSiteMmaSlot = 0x105,
  kSiteEpilogue = 0x106
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int per_b = p.tiles_i * p.tiles_j;
  bb = tile / per_b;
  const int r = tile - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <bool HAS_BIAS, bool HAS_MASK>
__global__ void __launch_bounds__(kThreads, 1) project_gate_kernel(const __grid_constant__ Params p) {
  constexpr uint32_t IDESC = idesc_f16_f32(128, 128, false, false);
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t w_bar, zfull[NSTAGE], zempty[NSTAGE], lnfull[NSTAGE];
  __shared__ __align__(8) uint64_t tfull[NSLOT], tempty[NSLOT], drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  float* par = reinterpret_cast<float*>(smem + OFF_PAR);  // [gamma 128 | beta 128 | bias 512]
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&w_bar, 1);
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&zfull[s], 1);
      mbar_init(&zempty[s], 1);
      mbar_init(&lnfull[s], 4);  // one arrival per LayerNorm warp
    }
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 4);  // one arrival per epilogue warp of the group that owns the slot
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  // Prologue (overlaps the previous kernel when launched with programmatic serialisation):
  // weights and parameters are never written by the kernels of this library, so they are
  // fetched before the dependency wait; z, mask, a, b and the status word only after it.
  for (int i = threadIdx.x; i < PAR_FLOATS; i += blockDim.x) {
    float v;
    if (i < CZ) v = __half2float(p.ln_w[i]);
    else if (i < 2 * CZ) v = __half2float(p.ln_b[i - CZ]);
    else v = HAS_BIAS ? p.bias[i - 2 * CZ] : 0.0f;
    par[i] = v;
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_z);
    tma_prefetch_desc(&p.tm_w);
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  if (warp == 0 && lane == 0) {
    mbar_arrive_expect_tx(&w_bar, NCH * WCHUNK_BYTES);
    for (int q = 0; q < NCH; ++q)
      for (int a = 0; a < KATOMS; ++a)
        tma_load_2d(smem + OFF_W + q * WCHUNK_BYTES + a * ATOM_BYTES, &p.tm_w, &w_bar, a * 64, q * 128);
  }
  griddep_trigger();
  griddep_wait();
  if (p.reset_status && blockIdx.x == 0 && threadIdx.x == 0) {
    p.status->code = 0;
    p.status->site = 0;
    p.status->block = 0;
  }

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        if (!mbar_wait(&zempty[s], ph ^ 1, ctx, kSiteProducer)) break;
        mbar_arrive_expect_tx(&zfull[s], A_BYTES);
        for (int a = 0; a < KATOMS; ++a)
          tma_load_4d(smem + OFF_A + s * A_BYTES + a * ATOM_BYTES, &p.tm_z, &zfull[s], a * 64, j0, i0, bb);
      }
      if (abort_sh) {
        mbar_drain(&w_bar, 0, 200000000ull);
        for (uint32_t s = 0; s < NSTAGE; ++s) {
          const uint32_t n_armed = it > s ? (it - s + 1) / 2 : 0;
          if (n_armed) mbar_drain(&zfull[s], (n_armed - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = mbar_wait(&w_bar, 0, ctx, kSiteMmaW);
      uint32_t it = 0, cit = 0;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        if (!mbar_wait(&lnfull[s], ph, ctx, kSiteMmaLn)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem + OFF_A + s * A_BYTES);
        for (int q = 0; q < NCH; ++q, ++cit) {
          const uint32_t slot = cit % NSLOT, sph = (cit / NSLOT) & 1;
          if (!mbar_wait(&tempty[slot], sph ^ 1, ctx, kSiteMmaSlot)) { ok = false; break; }
          tc_fence_after();
          const uint32_t w_base = smem_u32(smem + OFF_W + q * WCHUNK_BYTES);
#pragma unroll
          for (int kk = 0; kk < CZ / 16; ++kk) {
            const uint32_t off = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
            umma_f16(tmem_base + slot * 128, sdesc_sw128(a_base + off, 16, 1024), sdesc_sw128(w_base + off, 16, 1024),
                     IDESC, kk > 0 ? 1u : 0u);
          }
          umma_commit(&tfull[slot]);
        }
        umma_commit(&zempty[s]);  // the z/n tile may be refilled once these MMAs have read it
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < 6) {
    // ---------------- LayerNorm of the z tile, in place ----------------
    const int row = threadIdx.x - 64;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const uint32_t s = it & 1, ph = (it >> 1) & 1;
      if (!warp_wait(&zfull[s], ph, ctx, kSiteLn)) break;
      uint8_t* A = smem + OFF_A + s * A_BYTES;
      ln_row128_sw128(A, A, ATOM_BYTES, row, 1e-5f, LnParSmem{par, par + CZ});
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&lnfull[s]);
    }
  } else {
    // ---------------- epilogue: gate, mask, channel-major store ----------------
    const int ew = warp - 6;         // 0..11
    const int q = warp & 3;          // TMEM lane quadrant
    const int grp = ew >> 2;         // this warp drains the chunks with index % 3 == grp
    const int row = q * 32 + lane;   // position within the tile
    const int jo = (q * 32) % p.jw, io = (q * 32) / p.jw;  // this warp's 32 positions in the tile
    __half* stg = reinterpret_cast<__half*>(smem + OFF_STG + ew * 2 * WSTG_BYTES);
    constexpr bool has_bias = HAS_BIAS;
    constexpr bool has_mask = HAS_MASK;
    const float* bias = par + 2 * CZ;
    uint32_t cit = 0, sit = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const int gi = i0 + row / p.jw, gj = j0 + row % p.jw;
      float mval = 1.0f;
      if (HAS_MASK && gi < p.L && gj < p.L)
        mval = __half2float(p.mask[(static_cast<size_t>(bb) * p.L + gi) * p.L + gj]);
      const float2 m2 = make_float2(mval, mval);
      for (int qc = 0; qc < NCH; ++qc, ++cit) {
        if (cit % 3 != static_cast<uint32_t>(grp)) continue;
        const uint32_t slot = cit % NSLOT, sph = (cit / NSLOT) & 1;
        if (!warp_wait(&tfull[slot], sph, ctx, kSiteEpilogue)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + slot * 128;
        const int col0 = qc * 128;  // packed-row index of the chunk's first signal column
        const bool is_a = qc < NCH / 2;
        const int ch0 = (qc % (NCH / 2)) * 64;
#pragma unroll 1
        for (int sub = 0; sub < 64 / SUB; ++sub, ++sit) {
          uint32_t sg[16], gt[16];
          tmem_ld16(taddr + sub * SUB, sg);
          tmem_ld16(taddr + 64 + sub * SUB, gt);
          tmem_wait_ld16x2(sg, gt);
          if (sub == 64 / SUB - 1) {  // the whole slot has been read: hand it back to the MMA
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[slot]);
          }
          __half* st = stg + (sit & 1) * (WSTG_BYTES / 2);
          if (lane == 0) bulk_wait_read<1>();  // the store that last used this buffer has read it
          __syncwarp();
#pragma unroll
          for (int i = 0; i < SUB; i += 2) {
            float2 s = make_float2(__uint_as_float(sg[i]), __uint_as_float(sg[i + 1]));
            float2 g = make_float2(__uint_as_float(gt[i]), __uint_as_float(gt[i + 1]));
            if (has_bias) {
              const int c = col0 + sub * SUB + i;
              s = __fadd2_rn(s, make_float2(bias[c], bias[c + 1]));
              g = __fadd2_rn(g, make_float2(bias[c + 64], bias[c + 65]));
            }
            s = round_f16x2(s);  // proj is an fp16 tensor in the reference
            g = round_f16x2(g);
            float2 y = __fmul2_rn(s, sigmoid_f32x2(g));
            if (has_mask) y = __fmul2_rn(y, m2);
            st[i * 32 + lane] = __float2half_rn(y.x);
            st[(i + 1) * 32 + lane] = __float2half_rn(y.y);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(is_a ? &p.tm_a : &p.tm_b, st, j0 + jo, i0 + io, bb * CC + ch0 + sub * SUB);
            bulk_commit();
          }
        }
      }
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace k1
}  // namespace tmu
