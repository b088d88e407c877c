// K3W: K3 for c_z = c = 256 (mlx_trunk.py:4).  Same arithmetic as K3 (mlx_trunk.py:89-90,94-95;
// mlx_trunk_kernels.py:107-147,165-190,221-227):
//   m = fp16(LN_mix(x^T)), mixed = fp16(m @ w_emit [+ b]), g = fp16(n @ w_out_gate [+ b]),
//   z' = fp16(z + mixed * sigmoid(g)),  n = fp16(LN(z; norm_start)).
//
// w_emit and w_out_gate are 2 x 256 x 256 fp16 = 256 KB, more than shared memory, so each CTA
// owns one half of the OUTPUT channels (h = blockIdx.x mod 2; the grid is even) and keeps those
// 128 rows of both matrices resident (128 KB).  Both CTAs of a tile normalise the full 256-channel
// x column and z row (the LayerNorms are computed twice).  Because the sibling CTA reads all of
// z's channels while this one writes its half of z', z_out must not alias z (the host rejects it).
//
// One tile = 32 positions (small enough that every buffer is double-buffered next to the
// resident weights); D = W X^T with M = 128 output channels (TMEM lane = channel), N = 32
// positions, K = 256: emit into columns [0, 32) of a 64-column slot, gate into [32, 64).
// CTA = 14 warps, persistent:
//   warp 0      TMA: weights once; per tile the x tile (channel-major, 16 KB) and the z tile
//               (position-major, 128B-swizzled, 16 KB), 2 stages each
//   warp 1      TMEM (4 slots x 64 columns) + MMA thread
//   warps 2-5   A1 = fp16(LN_mix(x column)) over the x tile, one 64-channel atom per warp:
//               each thread gathers its row's 64 channels, the group meets, the rows are written
//               back K-major swizzled, the four partial sums are combined through shared memory.
//               With 1 x 32 tiles (XSW) the x tile arrives 64B-swizzled and each warp transposes
//               its atom with ldmatrix.trans (four lanes per position), combines the four atoms'
//               mean and M2 (parallel-variance formula) after one meeting, and writes A1 with
//               stmatrix: two group barriers per tile instead of four
//   warps 6-9   A2 = fp16(LN_in(z row)) into its own 2-stage buffer (z stays for the residual)
//   warps 10-13 epilogue, TMEM lane quadrant warp mod 4 (32 channels each): z' = z + m*sigmoid(g)
//               computed over the z tile's half-h atoms in shared memory, then TMA-stored.
#pragma once

#include "tmu_common.cuh"

namespace tmu {
namespace k3w {

constexpr int CZ = 256;
constexpr int CC = 256;
constexpr int TILE = 32;
constexpr int ATOM_BYTES = TILE * 128;          // activation atoms: 32 rows x 128 B
constexpr int WATOM_BYTES = 128 * 128;          // weight atoms: 128 rows x 128 B
constexpr int WBLOCK_BYTES = 128 * 256 * 2;     // 128 rows x K = 256
constexpr int TILE_BYTES = TILE * 256 * 2;      // 32 positions x 256 channels
constexpr int NSLOT = 4;
constexpr int OFF_WE = 0;
constexpr int OFF_WG = OFF_WE + WBLOCK_BYTES;
constexpr int OFF_X = OFF_WG + WBLOCK_BYTES;     // 2 stages: the x tile, then A1 in place
constexpr int OFF_Z = OFF_X + 2 * TILE_BYTES;    // 2 stages: the z tile, then z' (half h) in place
constexpr int OFF_A2 = OFF_Z + 2 * TILE_BYTES;   // 2 stages: LN_in(z)
constexpr int OFF_RED = OFF_A2 + 2 * TILE_BYTES; // float2 [2 groups][4 parts][32 rows]
constexpr int OFF_BAR = OFF_RED + 2 * 4 * TILE * 8;
constexpr int SMEM_BYTES = OFF_BAR + 256;
constexpr int kThreads = 448;
constexpr int TMEM_COLS = 256;
static_assert(SMEM_BYTES <= 232448, "K3W shared memory exceeds the per-block limit");

struct Params {
  CUtensorMap tm_z;   // z [B, rows, cols, 256]: box {64, jw, ih, 1}, 128B swizzle (load)
  CUtensorMap tm_zo;  // z_out, same geometry (store)
  CUtensorMap tm_x;   // x [B*256, rows, pitch]: box {jw, ih, 256}, no swizzle; XSW: box {32, 1, 256}, 64B swizzle
  CUtensorMap tm_we;  // w_emit [256, 256]: box {64, 128}
  CUtensorMap tm_wg;  // w_gate [256, 256]: box {64, 128}
  const __half* ln_in_w;
  const __half* ln_in_b;
  const __half* ln_mix_w;
  const __half* ln_mix_b;
  const float* b_emit;  // [256] or null
  const float* b_gate;  // [256] or null
  float mix_eps;
  int rows, cols, ih, jw, tiles_i, tiles_j, num_tiles;  // num_tiles = 2 x position tiles
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProdZ = 0x311, kSiteProdX = 0x312, kSiteMix = 0x313, kSiteIn = 0x314, kSiteMmaW = 0x315,
  kSiteMmaA = 0x316, kSiteMmaT = 0x317, kSiteEpilogue = 0x318
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int pt = tile >> 1;
  const int per_b = p.tiles_i * p.tiles_j;
  bb = pt / per_b;
  const int r = pt - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <bool HAS_BIAS, bool XSW>
__global__ void __launch_bounds__(kThreads, 1) emit_residual_w_kernel(const __grid_constant__ Params p) {
  const bool trace_on = trace_enabled(p.status);
  constexpr uint32_t IDESC = idesc_f16_f32(128, TILE, false, false);
  extern __shared__ uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(p.status, kStatusLayout, 0x31f);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t& w_bar = bars[0];
  uint64_t* xfull = bars + 1;
  uint64_t* xempty = bars + 3;
  uint64_t* zfull = bars + 5;
  uint64_t* zempty = bars + 7;
  uint64_t* a1full = bars + 9;
  uint64_t* a2full = bars + 11;
  uint64_t* a2empty = bars + 13;
  uint64_t* tfull = bars + 15;
  uint64_t* tempty = bars + 19;
  uint64_t& drain_bar = bars[23];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 24);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 24) + 4);
  volatile int* ok_sh = reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 25));  // [3]
  float2* red = reinterpret_cast<float2*>(smem + OFF_RED);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};
  const int hsel = blockIdx.x & 1;  // output channels [128 hsel, 128 hsel + 128); gridDim.x is even

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&w_bar, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);   // the MMA that read A1
      mbar_init(&zfull[s], 1);
      mbar_init(&zempty[s], 1);   // the epilogue's store of z' has read the stage
      mbar_init(&a1full[s], 4);   // the four LN_mix warps
      mbar_init(&a2full[s], 4);   // the four LN_in warps
      mbar_init(&a2empty[s], 1);  // the MMA that read A2
    }
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 4);
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
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  if (warp == 0 && lane == 0) {  // weights are never written by this library: load before the wait
    mbar_arrive_expect_tx(&w_bar, 2 * WBLOCK_BYTES);
    for (int a = 0; a < 4; ++a) {
      tma_load_2d(smem + OFF_WE + a * WATOM_BYTES, &p.tm_we, &w_bar, a * 64, hsel * 128);
      tma_load_2d(smem + OFF_WG + a * WATOM_BYTES, &p.tm_wg, &w_bar, a * 64, hsel * 128);
    }
  }
  griddep_trigger();
  griddep_wait();
  trace_mark_start(p.status, trace_on);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0, nz = 0, nx = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        if (!mbar_wait(&zempty[s], ph ^ 1, ctx, kSiteProdZ)) break;
        mbar_arrive_expect_tx(&zfull[s], TILE_BYTES);
        for (int a = 0; a < 4; ++a)
          tma_load_4d(smem + OFF_Z + s * TILE_BYTES + a * ATOM_BYTES, &p.tm_z, &zfull[s], a * 64, j0, i0, bb);
        ++nz;
        if (!mbar_wait(&xempty[s], ph ^ 1, ctx, kSiteProdX)) break;
        mbar_arrive_expect_tx(&xfull[s], TILE_BYTES);
        tma_load_3d(smem + OFF_X + s * TILE_BYTES, &p.tm_x, &xfull[s], j0, i0, bb * CC);
        ++nx;
      }
      if (abort_sh) {
        mbar_drain(&w_bar, 0, 200000000ull);
        for (uint32_t s = 0; s < 2; ++s) {
          const uint32_t nza = nz > s ? (nz - s + 1) / 2 : 0;
          if (nza) mbar_drain(&zfull[s], (nza - 1) & 1, 200000000ull);
          const uint32_t nxa = nx > s ? (nx - s + 1) / 2 : 0;
          if (nxa) mbar_drain(&xfull[s], (nxa - 1) & 1, 200000000ull);
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
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        const uint32_t slot = it & 3, sph = (it >> 2) & 1;
        if (!mbar_wait(&a1full[s], ph, ctx, kSiteMmaA)) break;
        if (!mbar_wait(&a2full[s], ph, ctx, kSiteMmaA)) break;
        if (!mbar_wait(&tempty[slot], sph ^ 1, ctx, kSiteMmaT)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + slot * 64;
        const uint64_t a1d = sdesc_sw128(smem_u32(smem + OFF_X + s * TILE_BYTES), 16, 1024);
        const uint64_t a2d = sdesc_sw128(smem_u32(smem + OFF_A2 + s * TILE_BYTES), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          const uint32_t ka = kk >> 2, kb = (kk & 3) * 32;
          umma_f16(d, sdesc_add(wed, ka * WATOM_BYTES + kb), sdesc_add(a1d, ka * ATOM_BYTES + kb), IDESC,
                   kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          const uint32_t ka = kk >> 2, kb = (kk & 3) * 32;
          umma_f16(d + TILE, sdesc_add(wgd, ka * WATOM_BYTES + kb), sdesc_add(a2d, ka * ATOM_BYTES + kb), IDESC,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(&xempty[s]);   // A1 has been read
        umma_commit(&a2empty[s]);  // A2 has been read
        umma_commit(&tfull[slot]);
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < 10) {
    // ---------------- LayerNorms: warps 2-5 LN_mix (x -> A1), warps 6-9 LN_in (z -> A2) ----------------
    const bool mix = warp < 6;
    const int grp = mix ? 0 : 1;
    const int t = threadIdx.x - (mix ? 64 : 192);
    const int row = t & 31, part = t >> 5;  // part = this warp's 64-channel atom
    const uint32_t bar_id = 1 + grp;
    float2* rd = red + grp * 4 * TILE;
    const LnParHalf par = mix ? LnParHalf{p.ln_mix_w, p.ln_mix_b} : LnParHalf{p.ln_in_w, p.ln_in_b};
    const float eps = mix ? p.mix_eps : 1e-5f;
    // XSW: this lane's LN_mix parameters, channel pairs 64 part + 32g + 8j + 2(t%4) (g < 2, j < 4)
    uint32_t gmw[8], bmw[8];
    if (XSW && mix) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = 64 * part + 32 * (e >> 2) + 8 * (e & 3) + 2 * (lane & 3);
        gmw[e] = __ldg(reinterpret_cast<const unsigned int*>(p.ln_mix_w + c));
        bmw[e] = __ldg(reinterpret_cast<const unsigned int*>(p.ln_mix_b + c));
      }
    }
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const uint32_t s = it & 1, ph = (it >> 1) & 1;
      // one thread waits (bounded) and shares the verdict, so the group meets at every barrier
      if (t == 0) {
        bool ok;
        if (mix) {
          ok = mbar_wait(&xfull[s], ph, ctx, kSiteMix);
        } else {
          ok = mbar_wait(&a2empty[s], ph ^ 1, ctx, kSiteIn);
          ok = ok && mbar_wait(&zfull[s], ph, ctx, kSiteIn);
        }
        ok_sh[grp] = ok ? 1 : 0;
      }
      named_bar_sync(bar_id, 128);
      if (!ok_sh[grp]) break;
      if (XSW && mix) {
        // The x tile: [channel][32 positions], 64 B per channel, the 16-byte chunk m (positions
        // 8m..8m+7) of channel ch at chunk m ^ ((ch >> 1) & 3).  ldmatrix.trans of the 8 x 8 block
        // (channels 8cb.., positions 8m..) gives lane t channels 8cb + 2(t%4), +1 of position
        // 8m + t/4 (lane t addresses channel 32g + t of this warp's atom; eight channel rows fall
        // in eight bank groups).
        const uint32_t xs = smem_u32(smem + OFF_X + s * TILE_BYTES);
        uint32_t u[4][8];  // u[m][4g + j]: channels 64 part + 32g + 8j + 2(t%4), +1 of position 8m + t/4
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const uint32_t ch = 64 * part + 32 * g + lane;
            ldsm_x4_trans(xs + ch * 64 + 16 * (m ^ ((ch >> 1) & 3)), u[m][4 * g], u[m][4 * g + 1], u[m][4 * g + 2],
                          u[m][4 * g + 3]);
          }
        // per position, this atom's mean and M2 (sum of squared deviations) around its own first
        // channel, from the four lanes that hold it
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float k = __shfl_sync(0xffffffffu, __low2float(*reinterpret_cast<const __half2*>(&u[m][0])), lane & ~3);
          float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            unsigned short lo, hi;
            split_half2(u[m][e], lo, hi);
            const float2 d = make_float2(add_f16_f32(lo, -k), add_f16_f32(hi, -k));
            s1 = __fadd2_rn(s1, d);
            s2 = __ffma2_rn(d, d, s2);
          }
          float t1 = s1.x + s1.y, t2 = s2.x + s2.y;
          t1 += __shfl_xor_sync(0xffffffffu, t1, 1);
          t2 += __shfl_xor_sync(0xffffffffu, t2, 1);
          t1 += __shfl_xor_sync(0xffffffffu, t1, 2);
          t2 += __shfl_xor_sync(0xffffffffu, t2, 2);
          if ((lane & 3) == 0) rd[part * TILE + 8 * m + (lane >> 2)] = make_float2(k + t1 * (1.0f / 64), t2 - t1 * t1 * (1.0f / 64));
        }
        named_bar_sync(bar_id, 128);  // every atom's partials are written; every x value is in registers
        uint8_t* A1 = smem + OFF_X + s * TILE_BYTES;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          // the four atoms combined (Chan et al.): mean of the means, M2 = sum M2_a + 64 sum (mean_a - mean)^2
          const int pos = 8 * m + (lane >> 2);
          const float2 a0 = rd[pos], a1 = rd[TILE + pos], a2 = rd[2 * TILE + pos], a3 = rd[3 * TILE + pos];
          const float mean = 0.25f * ((a0.x + a1.x) + (a2.x + a3.x));
          const float d0 = a0.x - mean, d1 = a1.x - mean, d2 = a2.x - mean, d3 = a3.x - mean;
          const float m2 = (a0.y + a1.y) + (a2.y + a3.y) + 64.0f * ((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3));
          const float rs = rsqrtf(fmaxf(m2 * (1.0f / 256), 0.0f) + eps);
          const float2 r2 = make_float2(rs, rs);
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              unsigned short lo, hi;
              split_half2(u[m][4 * g + j], lo, hi);
              const float2 d = __fmul2_rn(make_float2(add_f16_f32(lo, -mean), add_f16_f32(hi, -mean)), r2);
              const float2 gv = unpack_half2(gmw[4 * g + j]), bv = unpack_half2(bmw[4 * g + j]);
              const float2 y = __ffma2_rn(d, gv, bv);
              o[j] = pack_half2(y.x, y.y);
            }
            // A1 atom `part` (32 rows x 128 B, K-major 128B-swizzled): lane l gives the row of
            // position 8m + l%8 in chunk 4g + l/8
            const uint32_t row8 = lane & 7;
            stsm_x4(smem_u32(A1) + part * ATOM_BYTES + (8 * m + row8) * 128 + 16 * ((4 * g + (lane >> 3)) ^ row8), o[0], o[1],
                    o[2], o[3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a1full[s]);
        continue;
      }
      uint8_t* src;
      uint8_t* dst;
      if (mix) {
        // The x tile is [channel][position] (64 B per channel).  A1's atom a occupies exactly
        // the bytes of x channels [64a, 64a+64): gather this row's 64 channels of this warp's
        // atom, meet, and write them back as the swizzled K-major row.
        uint8_t* A = smem + OFF_X + s * TILE_BYTES;
        const __half* X = reinterpret_cast<const __half*>(A);
        uint32_t u[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int ch = 64 * part + 2 * k;
          __half2 h2 = __halves2half2(X[ch * TILE + row], X[(ch + 1) * TILE + row]);
          u[k] = *reinterpret_cast<uint32_t*>(&h2);
        }
        named_bar_sync(bar_id, 128);
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16)
          *reinterpret_cast<uint4*>(A + part * ATOM_BYTES + sw128_off(row, c16)) =
              make_uint4(u[4 * c16], u[4 * c16 + 1], u[4 * c16 + 2], u[4 * c16 + 3]);
        named_bar_sync(bar_id, 128);  // every row's channel 0 (the shift) is in place
        src = dst = A;
      } else {
        src = smem + OFF_Z + s * TILE_BYTES;
        dst = smem + OFF_A2 + s * TILE_BYTES;
      }
      const float shift = ln_row_shift(src, row);
      rd[part * TILE + row] = ln_atom_sums(src, ATOM_BYTES, row, part, shift);
      named_bar_sync(bar_id, 128);
      const float2 s0 = rd[row], s1 = rd[TILE + row], s2 = rd[2 * TILE + row], s3 = rd[3 * TILE + row];
      const float2 mr = ln256_moments(make_float2(s0.x + s1.x, s0.y + s1.y), make_float2(s2.x + s3.x, s2.y + s3.y),
                                      shift, eps);
      ln_atom_apply(src, dst, ATOM_BYTES, row, part, mr.x, mr.y, par);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(mix ? &a1full[s] : &a2full[s]);
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;                       // TMEM lane quadrant this warp may access
    const int ch = hsel * 128 + q * 32 + lane;    // this thread's output channel
    const uint32_t zoff = (ch >> 6) * ATOM_BYTES + (ch & 7) * 2;  // + sw128_off(position, chunk)
    const uint32_t chunk = (ch & 63) >> 3;
    float be = 0.f, bgv = 0.f;
    if (HAS_BIAS) {
      be = __ldg(p.b_emit + ch);
      bgv = __ldg(p.b_gate + ch);
    }
    const float2 be2 = make_float2(be, be), bg2 = make_float2(bgv, bgv);
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t s = it & 1, ph = (it >> 1) & 1;
      const uint32_t slot = it & 3, sph = (it >> 2) & 1;
      if (warp == 10 && lane == 0) {
        bool ok = mbar_wait(&tfull[slot], sph, ctx, kSiteEpilogue);
        ok = ok && mbar_wait(&zfull[s], ph, ctx, kSiteEpilogue);
        ok_sh[2] = ok ? 1 : 0;
      }
      named_bar_sync(3, 128);
      if (!ok_sh[2]) break;
      tc_fence_after();
      uint8_t* Zs = smem + OFF_Z + s * TILE_BYTES;
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + slot * 64;
#pragma unroll 1
      for (int pb = 0; pb < TILE; pb += 16) {
        uint32_t em[16], gt[16];
        tmem_ld16(trow + pb, em);
        tmem_ld16(trow + TILE + pb, gt);
        tmem_wait_ld16x2(em, gt);
        if (pb == TILE - 16) {  // the slot has been read: hand it back to the MMA
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[slot]);
        }
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          __half* z0 = reinterpret_cast<__half*>(Zs + zoff + sw128_off(pb + i, chunk));
          __half* z1 = reinterpret_cast<__half*>(Zs + zoff + sw128_off(pb + i + 1, chunk));
          float2 m = make_float2(__uint_as_float(em[i]), __uint_as_float(em[i + 1]));
          float2 g = make_float2(__uint_as_float(gt[i]), __uint_as_float(gt[i + 1]));
          if (HAS_BIAS) {
            m = __fadd2_rn(m, be2);
            g = __fadd2_rn(g, bg2);
          }
          m = round_f16x2(m);  // mixed and g are fp16 tensors in the reference
          g = round_f16x2(g);
          const float2 zn = __ffma2_rn(m, sigmoid_f32x2(g), make_float2(__half2float(*z0), __half2float(*z1)));
          *z0 = __float2half_rn(zn.x);
          *z1 = __float2half_rn(zn.y);
        }
      }
      fence_proxy_async_smem();  // z' (generic-proxy writes) -> visible to the TMA store
      named_bar_sync(3, 128);
      if (warp == 10 && lane == 0) {
        for (int k = 0; k < 2; ++k) {
          const int a = 2 * hsel + k;
          tma_store_4d(&p.tm_zo, Zs + a * ATOM_BYTES, a * 64, j0, i0, bb);
        }
        bulk_commit();
        bulk_wait_read<0>();
        mbar_arrive(&zempty[s]);
      }
    }
    if (warp == 10 && lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  trace_mark_end(p.status, trace_on);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace k3w
}  // namespace tmu
