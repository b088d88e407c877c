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
// One tile = 128 positions (ih x jw block).  CTA = 23 warps, one per SM, persistent:
//   warp 0     TMA: w_emit and w_gate once (resident), then per tile the z tile (3 stages,
//              128B-swizzled position-major); warp 22 the x tile (2 stages, channel-major)
//   warp 1     TMEM (2 x 256 columns) + MMA thread: emit (A1 x W_e) and gate (A2 x W_g)
//   warps 2-9  A1 = fp16(LN_mix(x column)), written over the x tile it was gathered from once
//              every thread holds its part of the columns in registers.  With jw >= 64 (XMODE
//              1) the x tile arrives as two 128B-swizzled [channel][64 positions] halves, with
//              jw == 32 (XMODE 2) as four 64B-swizzled [channel][32 positions] quarters, and is
//              transposed by ldmatrix.trans (four lanes per position, conflict-free), A1
//              written by stmatrix; otherwise a lane pair per position gathers 2-byte values;
//   warps 10-13 A2 = fp16(LN_in(z row)), in place over the z stage; both concurrently, both
//              K-major 128B-swizzled UMMA operands.  A2 in place (instead of one separate A2
//              buffer) lets LN_in run ahead of the MMA, and its 32 KB pays for a third z stage;
//              after the MMA has read A2, warp 22 reloads the tile's z into the stage (an L2
//              hit) for the residual, ahead of the epilogue.
//   warps 14-21 epilogue, two groups of four warps (one per TMEM lane quadrant); group h owns
//              output channels [64h, 64h+64): TMEM -> gate/residual in fp32 -> z' written over
//              the z tile -> each warp TMA-stores its own 32 positions x 64 channels
//   warp 22    TMA: the x tiles (warp 0 keeps the z tiles), so an x load never queues behind
//              the z stage, which stays busy until the epilogue has stored z'; and the residual
//              reloads, one tile behind the x loads
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
constexpr int NZ = 3;                          // z stages: z, then A2 in place, then z again
constexpr int OFF_Z = OFF_WG + CZ * CZ * 2;
constexpr int OFF_X = OFF_Z + NZ * TILE_BYTES;   // 2 stages; stage s holds the x tile, then A1 in place
constexpr int OFF_PAR = OFF_X + 2 * TILE_BYTES;  // fp32 LN params: in gamma, in beta, mix gamma, mix beta
constexpr int OFF_BAR = OFF_PAR + 4 * 128 * 4;   // mbarriers and flags
constexpr int SMEM_BYTES = OFF_BAR + 512;        // no alignment slack: the kernel checks the base instead
static_assert(SMEM_BYTES <= 232448, "K3 shared memory exceeds the per-block limit");
constexpr int kThreads = 736;
constexpr int TMEM_COLS = 512;

struct Params {
  CUtensorMap tm_z;   // z [B, rows, cols, c_z]: box {64, jw, ih, 1}, 128B swizzle (load)
  CUtensorMap tm_zo;  // z_out: box {64, min(jw,32), 32/min(jw,32), 1}, 128B swizzle (per-warp store)
  CUtensorMap tm_x;   // x [B*c, L, Lpad]: box {jw, ih, c}, no swizzle; XMODE 1: box {64, 1, c}, 128B
                      // swizzle; XMODE 2: box {32, 1, c}, 64B swizzle
  CUtensorMap tm_we;  // w_emit [c_z, c]: box {64, 128}
  CUtensorMap tm_wg;  // w_gate [c_z, c_z]: box {64, 128}
  const __half* ln_in_w;
  const __half* ln_in_b;
  const __half* ln_mix_w;
  const __half* ln_mix_b;
  const float* b_emit;  // [c_z] or null
  const float* b_gate;  // [c_z] or null
  float mix_eps;
  int rows, cols, ih, jw, tiles_i, tiles_j, num_tiles;
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProdZ = 0x301, kSiteProdX = 0x302, kSiteTrA = 0x303, kSiteTrX = 0x304, kSiteTrZ = 0x305,
  kSiteMmaW = 0x306, kSiteMmaA = 0x307, kSiteMmaT = 0x308, kSiteEpilogue = 0x309, kSiteProdR = 0x30a
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int per_b = p.tiles_i * p.tiles_j;
  bb = tile / per_b;
  const int r = tile - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <bool HAS_BIAS, int XMODE>
__global__ void __launch_bounds__(kThreads, 1) emit_residual_kernel(const __grid_constant__ Params p) {
  const bool trace_on = trace_enabled(p.status);
  constexpr uint32_t IDESC = idesc_f16_f32(128, CZ, false, false);
  // All shared state lives in the dynamic buffer (no static __shared__), whose base the 128B
  // swizzle needs 1024-byte aligned; a misaligned base is reported, never computed on.
  extern __shared__ uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(p.status, kStatusLayout, 0x3ff);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t& w_bar = bars[0];
  uint64_t* zfull = bars + 1;       // [NZ] z loaded
  uint64_t* zempty = bars + 4;      // [NZ] the epilogue's stores have read z'
  uint64_t* xfull = bars + 7;       // [2]
  uint64_t* xempty = bars + 9;      // [2] committed by the MMA that read A1 from this stage
  uint64_t* a2full = bars + 11;     // [NZ] A2 written in place over z stage s (the four LN_in warps)
  uint64_t* zread = bars + 14;      // [NZ] committed by the MMA that read A2 from z stage s
  uint64_t* rfull = bars + 17;      // [NZ][2] z atom h reloaded into stage s for the epilogue
  uint64_t* tfull = bars + 23;      // [2]
  uint64_t* tempty = bars + 25;     // [2]
  uint64_t* a1full = bars + 27;     // [2] A1 written over x stage s (the eight LN_mix warps)
  uint64_t& drain_bar = bars[29];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 30);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 30) + 4);
  volatile int& x_ok_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 31));
  volatile int* gflags = reinterpret_cast<volatile int*>(bars + 32);  // [3 groups][2] group_wait verdicts
  float* par = reinterpret_cast<float*>(smem + OFF_PAR);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&w_bar, 1);
    for (int s = 0; s < NZ; ++s) {
      mbar_init(&zfull[s], 1);
      mbar_init(&zempty[s], 8);   // each epilogue warp, once its store has read the tile
      mbar_init(&a2full[s], 4);   // the four LN_in warps
      mbar_init(&zread[s], 1);
      mbar_init(&rfull[2 * s], 1);
      mbar_init(&rfull[2 * s + 1], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 8);   // one arrival per epilogue warp
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
      // A1 and A2 have separate barriers: LN_mix may finish tile t+1 before LN_in finishes tile t
      mbar_init(&a1full[s], 8);   // the eight LN_mix warps
    }
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
  for (int i = threadIdx.x; i < 4 * 128; i += blockDim.x) {
    if (XMODE != 0 && i >= 256) {  // mix parameters interleaved per channel pair: {g[2k], g[2k+1], b[2k], b[2k+1]}
      const int k = (i - 256) >> 2, e = i & 3;
      par[i] = __half2float(e < 2 ? p.ln_mix_w[2 * k + e] : p.ln_mix_b[2 * k + e - 2]);
    } else {
      const __half* src = i < 128 ? p.ln_in_w : i < 256 ? p.ln_in_b : i < 384 ? p.ln_mix_w : p.ln_mix_b;
      par[i] = __half2float(src[i & 127]);
    }
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  // weights are never written by this library's kernels: fetch them before the dependency wait
  if (warp == 0 && lane == 0) {
    mbar_arrive_expect_tx(&w_bar, (CZ * CC + CZ * CZ) * 2);
    for (int a = 0; a < CC / 64; ++a) tma_load_2d(smem + OFF_WE + a * ATOM_BYTES, &p.tm_we, &w_bar, a * 64, 0);
    for (int a = 0; a < CZ / 64; ++a) tma_load_2d(smem + OFF_WG + a * ATOM_BYTES, &p.tm_wg, &w_bar, a * 64, 0);
  }
  griddep_trigger();
  griddep_wait();  // x, z come from previous kernels; z_out may alias what they read
  trace_mark_start(p.status, trace_on);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // z tiles; the x tiles have their own producer (warp 22), so an x load never waits
      // behind the long-lived z stage (held until the epilogue has stored z')
      uint32_t it = 0, nz = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const uint32_t s = it % NZ, ph = (it / NZ) & 1;
        if (!mbar_wait(&zempty[s], ph ^ 1, ctx, kSiteProdZ)) break;
        mbar_arrive_expect_tx(&zfull[s], TILE_BYTES);
        for (int a = 0; a < CZ / 64; ++a)
          tma_load_4d(smem + OFF_Z + s * TILE_BYTES + a * ATOM_BYTES, &p.tm_z, &zfull[s], a * 64, j0, i0, bb);
        ++nz;
      }
      if (abort_sh) {
        mbar_drain(&w_bar, 0, 200000000ull);
        for (uint32_t s = 0; s < NZ; ++s) {
          const uint32_t nza = nz > s ? (nz - s + NZ - 1) / NZ : 0;
          if (nza) mbar_drain(&zfull[s], (nza - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 22) {
    // ---------------- TMA producer: x tiles and the residual reloads ----------------
    // After the MMA has read A2 from a z stage (zread), the stage is refilled with that tile's z
    // (an L2 hit) for the epilogue's residual.  The reload of tile t is issued here, right after
    // the x load of tile t + 1: both wait for the same MMA commits (xempty of the stage x(t + 1)
    // reuses and zread of t come from the MMAs of t - 1 and t), so neither waits on the other,
    // and the reload is in flight while the epilogue is still busy with tile t - 1.
    if (lane == 0) {
      uint32_t it = 0, nx = 0, nr = 0;
      int pb = 0, pi = 0, pj = 0;  // the previous tile, whose reload is due
      auto reload = [&](uint32_t k, int bb, int i0, int j0) -> bool {
        const uint32_t s = k % NZ, ph = (k / NZ) & 1;
        if (!mbar_wait(&zread[s], ph, ctx, kSiteProdR)) return false;
        for (int h = 0; h < 2; ++h) {
          mbar_arrive_expect_tx(&rfull[2 * s + h], ATOM_BYTES);
          tma_load_4d(smem + OFF_Z + s * TILE_BYTES + h * ATOM_BYTES, &p.tm_z, &rfull[2 * s + h], h * 64, j0, i0, bb);
        }
        ++nr;
        return true;
      };
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        if (!mbar_wait(&xempty[s], ph ^ 1, ctx, kSiteProdX)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&xfull[s], TILE * CC * 2);
        if (XMODE == 1) {  // positions 0-63, then 64-127 (the tile's second half-row, or its second row)
          tma_load_3d(smem + OFF_X + s * TILE_BYTES, &p.tm_x, &xfull[s], j0, i0, bb * CC);
          tma_load_3d(smem + OFF_X + s * TILE_BYTES + TILE_BYTES / 2, &p.tm_x, &xfull[s], p.jw == 128 ? j0 + 64 : j0,
                      p.jw == 128 ? i0 : i0 + 1, bb * CC);
        } else if (XMODE == 2) {  // the tile's four rows of 32 positions
          for (int r = 0; r < 4; ++r)
            tma_load_3d(smem + OFF_X + s * TILE_BYTES + r * (TILE_BYTES / 4), &p.tm_x, &xfull[s], j0, i0 + r, bb * CC);
        } else {
          tma_load_3d(smem + OFF_X + s * TILE_BYTES, &p.tm_x, &xfull[s], j0, i0, bb * CC);
        }
        ++nx;
        if (it > 0 && !reload(it - 1, pb, pi, pj)) {
          ok = false;
          break;
        }
        pb = bb, pi = i0, pj = j0;
      }
      if (ok && it > 0) reload(it - 1, pb, pi, pj);
      if (abort_sh) {
        for (uint32_t s = 0; s < 2; ++s) {
          const uint32_t nxa = nx > s ? (nx - s + 1) / 2 : 0;
          if (nxa) mbar_drain(&xfull[s], (nxa - 1) & 1, 200000000ull);
        }
        for (uint32_t s = 0; s < NZ; ++s) {  // reloads in flight land before the CTA exits
          const uint32_t nra = nr > s ? (nr - s + NZ - 1) / NZ : 0;
          if (nra) {
            mbar_drain(&rfull[2 * s], (nra - 1) & 1, 200000000ull);
            mbar_drain(&rfull[2 * s + 1], (nra - 1) & 1, 200000000ull);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = mbar_wait(&w_bar, 0, ctx, kSiteMmaW);
      uint32_t it = 0;
      const uint64_t wed = sdesc_sw128(smem_u32(smem + OFF_WE), 16, 1024), wgd = sdesc_sw128(smem_u32(smem + OFF_WG), 16, 1024);
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
        const uint32_t acc = it & 1, aph = (it >> 1) & 1;
        const uint32_t zs = it % NZ, zph = (it / NZ) & 1;
        if (!mbar_wait(&a1full[it & 1], (it >> 1) & 1, ctx, kSiteMmaA)) break;
        if (!mbar_wait(&a2full[zs], zph, ctx, kSiteMmaA)) break;
        const uint32_t a2 = smem_u32(smem + OFF_Z + zs * TILE_BYTES);
        if (!mbar_wait(&tempty[acc], aph ^ 1, ctx, kSiteMmaT)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * 256;
        const uint32_t a1 = smem_u32(smem + OFF_X + (it & 1) * TILE_BYTES);
        const uint64_t a1d = sdesc_sw128(a1, 16, 1024), a2d = sdesc_sw128(a2, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < CC / 16; ++kk) {
          const uint32_t off = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
          umma_f16(d, sdesc_add(a1d, off), sdesc_add(wed, off), IDESC, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < CZ / 16; ++kk) {
          const uint32_t off = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
          umma_f16(d + CZ, sdesc_add(a2d, off), sdesc_add(wgd, off), IDESC, kk > 0 ? 1u : 0u);
        }
        umma_commit(&xempty[it & 1]);  // A1 (over the x tile) and A2 (over the z tile) have been read
        umma_commit(&zread[zs]);
        umma_commit(&tfull[acc]);
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < 10) {
    // ---------------- A1 = LN_mix of each position's x column (a lane pair per position) ----------------
    const int row = (threadIdx.x - 64) >> 1, half = threadIdx.x & 1;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const uint32_t s = it & 1, ph = (it >> 1) & 1;
      // one thread waits (bounded) and shares the verdict, so the eight warps always meet at
      // the named barriers below together
      if (threadIdx.x == 64) x_ok_sh = mbar_wait(&xfull[s], ph, ctx, kSiteTrX) ? 1 : 0;
      named_bar_sync(1, 256);
      if (!x_ok_sh) break;
      if constexpr (XMODE != 0) {
        // The x stage holds two halves of 64 tile positions, each [channel][64 positions] with
        // 128 B per channel and the 16-byte chunk m (positions 8m..8m+7) at chunk m ^ (channel
        // & 7).  Warp wl owns tile positions [16 wl, 16 wl + 16) = chunks m0, m0 + 1 of half
        // wl / 4.  ldmatrix.trans of the 8 x 8 block (channels 8cb.., positions 8m..) gives lane
        // t channels 8cb + 2(t%4), +1 of position 8m + t/4: four lanes per position, 32
        // channels each; lane t supplies the row address of channel 32q + t.
        // XMODE 2: four quarters [channel][32 positions], 64 B per channel, chunk m of channel ch
        // at chunk m ^ ((ch >> 1) & 3); warp wl's positions are chunks m0, m0 + 1 of quarter wl / 2.
        const int wl = warp - 2;
        const uint32_t xs = smem_u32(smem + OFF_X + s * TILE_BYTES);
        const uint32_t xh = XMODE == 1 ? xs + (wl >> 2) * (TILE_BYTES / 2) : xs + (wl >> 1) * (TILE_BYTES / 4);
        const int m0 = XMODE == 1 ? 2 * (wl & 3) : 2 * (wl & 1);
        uint32_t u[2][16];  // u[mi][4q + j]: channels 32q + 8j + 2(t%4), +1 of position 16 wl + 8 mi + t/4
#pragma unroll
        for (int mi = 0; mi < 2; ++mi)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t ch = 32 * q + lane;
            const uint32_t addr = XMODE == 1 ? xh + ch * 128 + 16 * ((m0 + mi) ^ (lane & 7))
                                             : xh + ch * 64 + 16 * ((m0 + mi) ^ ((ch >> 1) & 3));
            ldsm_x4_trans(addr, u[mi][4 * q], u[mi][4 * q + 1], u[mi][4 * q + 2], u[mi][4 * q + 3]);
          }
        // statistics of each position over its four lanes: shifted sums around its channel 0
        // (the low half of u[mi][0] on lane t with t%4 == 0), two shuffle steps
        float mean[2], rs[2];
#pragma unroll
        for (int mi = 0; mi < 2; ++mi) {
          const float kshift =
              __shfl_sync(0xffffffffu, __low2float(*reinterpret_cast<const __half2*>(&u[mi][0])), lane & ~3);
          float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            unsigned short lo, hi;
            split_half2(u[mi][k], lo, hi);
            const float2 d = make_float2(add_f16_f32(lo, -kshift), add_f16_f32(hi, -kshift));
            s1 = __fadd2_rn(s1, d);
            s2 = __ffma2_rn(d, d, s2);
          }
          float t1 = s1.x + s1.y, t2 = s2.x + s2.y;
          t1 += __shfl_xor_sync(0xffffffffu, t1, 1);
          t2 += __shfl_xor_sync(0xffffffffu, t2, 1);
          t1 += __shfl_xor_sync(0xffffffffu, t1, 2);
          t2 += __shfl_xor_sync(0xffffffffu, t2, 2);
          const float m1 = t1 * (1.0f / 128);
          const float var = fmaxf(t2 * (1.0f / 128) - m1 * m1, 0.0f);
          mean[mi] = kshift + m1;
          rs[mi] = rsqrtf(var + p.mix_eps);
        }
        named_bar_sync(1, 256);  // every x value is in registers: overwrite the tile with A1
        // A1 (K-major, 128B-swizzled atoms of 64 channels): stmatrix of the same 8 x 8 blocks,
        // rows = positions; lane t supplies the row address of position 16 wl + 8 mi + t%8 in
        // chunk 4(q%2) + t/8 of atom q/2.
        const float4* mp = reinterpret_cast<const float4*>(par + 256);  // interleaved per channel pair
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float4 gb[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) gb[j] = mp[16 * q + 4 * j + (lane & 3)];
#pragma unroll
          for (int mi = 0; mi < 2; ++mi) {
            const float2 r2 = make_float2(rs[mi], rs[mi]);
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              unsigned short lo, hi;
              split_half2(u[mi][4 * q + j], lo, hi);
              const float2 d = __fmul2_rn(make_float2(add_f16_f32(lo, -mean[mi]), add_f16_f32(hi, -mean[mi])), r2);
              const float2 y = __ffma2_rn(d, make_float2(gb[j].x, gb[j].y), make_float2(gb[j].z, gb[j].w));
              o[j] = pack_half2(y.x, y.y);
            }
            const uint32_t pos = 16 * wl + 8 * mi + (lane & 7);
            stsm_x4(xs + (q >> 1) * ATOM_BYTES + pos * 128 + 16 * ((4 * (q & 1) + (lane >> 3)) ^ (lane & 7)), o[0], o[1],
                    o[2], o[3]);
          }
        }
      } else {
        // The x tile is [channel][position] (256 B per channel).  A1's 64-channel atom h occupies
        // exactly the bytes of x channels [64h, 64h+64): each thread gathers its half of this
        // position's column into registers, the pair computes the row's statistics, the 256
        // threads meet, and each writes its normalised half as row `row` of atom `half` of the
        // K-major swizzled A1 operand.
        const __half* X = reinterpret_cast<const __half*>(smem + OFF_X + s * TILE_BYTES);
        uint8_t* A1 = smem + OFF_X + s * TILE_BYTES;
        uint32_t u[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int ch = 64 * half + 2 * k;
          __half2 h2 = __halves2half2(X[ch * TILE + row], X[(ch + 1) * TILE + row]);
          u[k] = *reinterpret_cast<uint32_t*>(&h2);
        }
        // LayerNorm of the row straight from the two lanes' registers: statistics as shifted sums
        // around the row's channel 0 (held by the half-0 lane), combined with one shuffle, then the
        // normalised half written once, over the x bytes every thread has finished reading.
        const float kshift = __shfl_sync(0xffffffffu, __low2float(*reinterpret_cast<const __half2*>(&u[0])), lane & ~1);
        float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          unsigned short lo, hi;
          split_half2(u[k], lo, hi);
          const float2 d = make_float2(add_f16_f32(lo, -kshift), add_f16_f32(hi, -kshift));
          s1 = __fadd2_rn(s1, d);
          s2 = __ffma2_rn(d, d, s2);
        }
        float t1 = s1.x + s1.y, t2 = s2.x + s2.y;
        t1 += __shfl_xor_sync(0xffffffffu, t1, 1);
        t2 += __shfl_xor_sync(0xffffffffu, t2, 1);
        const float m1 = t1 * (1.0f / 128);
        const float var = fmaxf(t2 * (1.0f / 128) - m1 * m1, 0.0f);
        const float mean = kshift + m1;
        const float rs = rsqrtf(var + p.mix_eps);
        const float2 r2 = make_float2(rs, rs);
        const LnParSmem mpar{par + 256, par + 384};
        named_bar_sync(1, 256);  // every column half is in registers: overwrite the tile
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 8 channels 64 half + 8c .. at a time
          float g[8], b[8];
          mpar(8 * half + c, g, b);
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            unsigned short lo, hi;
            split_half2(u[4 * c + e], lo, hi);
            const float2 d = __fmul2_rn(make_float2(add_f16_f32(lo, -mean), add_f16_f32(hi, -mean)), r2);
            const float2 y = __ffma2_rn(d, make_float2(g[2 * e], g[2 * e + 1]), make_float2(b[2 * e], b[2 * e + 1]));
            o[e] = pack_half2(y.x, y.y);
          }
          *reinterpret_cast<uint4*>(A1 + half * ATOM_BYTES + sw128_off(row, c)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a1full[s]);
    }
  } else if (warp < 14) {
    // ---------------- A2 = LN_in of each position's z row ----------------
    const int row = threadIdx.x - 320;
    uint32_t it = 0, gcount = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const uint32_t s = it % NZ, ph = (it / NZ) & 1;
      if (!group_wait(&zfull[s], ph, nullptr, 0, ctx, kSiteTrZ, row == 0, 2, 128, gflags, gcount)) break;
      uint8_t* Z = smem + OFF_Z + s * TILE_BYTES;
      ln_row128_sw128(Z, Z, ATOM_BYTES, row, 1e-5f, LnParSmem{par, par + 128});  // A2 in place
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a2full[s]);
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;          // TMEM lane quadrant
    const int h = (warp - 14) >> 2;  // output channels [64h, 64h+64)
    const int row = q * 32 + lane;
    const int jo = (q * 32) % p.jw, io = (q * 32) / p.jw;  // this warp's 32 positions in the tile
    constexpr bool has_be = HAS_BIAS, has_bg = HAS_BIAS;
    uint32_t it = 0, gcount = 0;
    const bool leader = ((warp - 14) & 3) == 0 && lane == 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t s = it % NZ, ph = (it / NZ) & 1;
      const uint32_t acc = it & 1, aph = (it >> 1) & 1;
      uint8_t* Zh = smem + OFF_Z + s * TILE_BYTES + h * ATOM_BYTES;
      // the accumulators and this half's z atom, reloaded for the residual by warp 22; one thread
      // of each channel half's four warps waits, the others park on barrier 3 + h
      if (!group_wait(&tfull[acc], aph, &rfull[2 * s + h], ph, ctx, kSiteEpilogue, leader, 3 + h, 128,
                      gflags + 2 + 2 * h, gcount))
        break;
      tc_fence_after();
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * 256 + h * 64;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {  // 16 output channels at a time
        uint32_t em[16], gt[16];
        tmem_ld16(trow + cc * 16, em);
        tmem_ld16(trow + CZ + cc * 16, gt);
        tmem_wait_ld16x2(em, gt);
        if (cc == 3) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint8_t* zp = Zh + sw128_off(row, cc * 2 + j);
          uint4 zv = *reinterpret_cast<const uint4*>(zp);
          uint32_t* zu = reinterpret_cast<uint32_t*>(&zv);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int i = j * 8 + k * 2;
            const int n = h * 64 + cc * 16 + i;
            float2 m = make_float2(__uint_as_float(em[i]), __uint_as_float(em[i + 1]));
            float2 g = make_float2(__uint_as_float(gt[i]), __uint_as_float(gt[i + 1]));
            if (has_be) m = __fadd2_rn(m, __ldg(reinterpret_cast<const float2*>(p.b_emit + n)));
            if (has_bg) g = __fadd2_rn(g, __ldg(reinterpret_cast<const float2*>(p.b_gate + n)));
            m = round_f16x2(m);  // mixed and g are fp16 tensors in the reference
            g = round_f16x2(g);
            const float2 zn = __ffma2_rn(m, sigmoid_f32x2(g), unpack_half2(zu[k]));
            zu[k] = pack_half2(zn.x, zn.y);
          }
          *reinterpret_cast<uint4*>(zp) = zv;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_4d(&p.tm_zo, Zh + q * 32 * 128, h * 64, j0 + jo, i0 + io, bb);
        bulk_commit();
        bulk_wait_read<0>();
        mbar_arrive(&zempty[s]);
      }
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  trace_mark_end(p.status, trace_on);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace k3
}  // namespace tmu
