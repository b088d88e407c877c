// K4: the pair transition of a PairUpdateBlock, z' = z + ffn(LN(z)), in one pass over the pair
// grid (c_z = 128 or 256, hidden h a multiple of 64).
//
// Reference (src/esmfold2_mlx/): mlx_trunk.py:96-99, fused path mlx_trunk_kernels.py:236-239
// (module form fast_trunk.py:35-42), in the fp16 scheme:
//   h  = fp16(LN(z; norm, eps=1e-5))
//   x  = fp16(h @ w12^T)                       w12 [2h, c_z] (SwiGLU) or [h, c_z] (ReLU)
//   SwiGLU: s = fp16(fp16(x1 * fp16(sigmoid(x1))) * x2),  x1 = x[:, :h], x2 = x[:, h:]
//   ReLU (synthetic configurations only): s = relu(x)
//   z' = fp16(z + s @ w3^T)                    w3 [c_z, h]; one rounding (mx.addmm)
//
// Tile = 128 positions (ih x jw block of the grid); TMEM lane = position.  The hidden dimension
// is processed in chunks: GEMM1 of chunk k (D1 = h W12_k^T, N = 128: for SwiGLU a chunk is 64
// hidden units, the B operand stacking its 64 x1 rows over its 64 x2 rows; for ReLU a chunk is
// 128 hidden units, its first 64 rows over its next 64, so GEMM1 is N = 128 MMAs, which one
// issuing thread drives at the tensor core's rate where N = 64 MMAs reach about two thirds of
// it) lands in one of two TMEM chunk buffers, the activation warps turn it into the fp16 A
// operand s in shared memory (SwiGLU: one 64-wide s per chunk; ReLU: two, one per s buffer),
// and GEMM2 accumulates D2 += s W3^T (N = c_z as 128-column MMAs, K = 64 per s) in a per-tile
// TMEM accumulator.  The MMA thread issues G1(0), G1(1), G1(2), G2(0), G1(3), G2(1), ...
// (GEMM1 two chunks ahead), so the tensor core computes the next chunks while the current ones
// are being activated.  The weights (256 KB - 1.5 MB) do not fit beside the tiles, so they
// stream from L2 through a 4-stage ring of 16 KB items in exactly that order.
//
// c_z = 128: z tiles (2 stages) and LayerNorm outputs h (2 stages) are separate buffers, and the
// epilogue adds D2 to the z tile still in shared memory; two D2 accumulators (256 columns).
// c_z = 256: a 64 KB tile leaves room for two tile buffers only, so each holds z, is normalised
// in place into h, and after the tile's last GEMM1 is refilled with z (an L2 hit: the same CTA
// read it microseconds before) for the epilogue; one 256-column D2 accumulator.
// CTA = 19 warps, one per SM, persistent:
//   warp 0      TMA: the weight ring
//   warp 1      TMEM (512 columns: D2 at [0, 256), D1 x 2 at [256, 512)) + MMA thread
//   warp 2      TMA: z tiles (2 stages)
//   warps 3-6   LayerNorm z tile -> h (K-major swizzled A operand, 2 stages)
//   warps 7-14  activation: D1 -> s, two groups of four (one TMEM lane quadrant per warp),
//               group g on the chunks that use buffer g
//   warps 15-18 epilogue: D2 + z -> z' over the z tile, per-warp TMA store of 32 positions
// Each tile is read and written by exactly one CTA, so z_out may alias z.
//
// h mode (MODE == kModeH): the transition layers of the diffusion head's pair conditioning
// (mlx_diffusion16.py:64-67,83-84: z = z + fp32(fp16(silu(h@a) * (h@b)) @ out), h = fp16(LN(z)),
// the residual stream fp32).  h comes precomputed from the row LayerNorm pass (which rebuilds
// the fp32 z from its fp16 terms) and is loaded by TMA straight into the A-operand stages; the
// epilogue stores only t = fp16(D2), the next term of z.  The SwiGLU arithmetic (w12 = [a; b]
// rows) is the trunk transition's.
#pragma once

#include "ln_rows.cuh"

namespace tmu {
namespace k4 {

constexpr int TILE = 128;
constexpr int CHUNK = 64;                        // hidden units per s buffer (a SwiGLU chunk; half a ReLU chunk)
constexpr int ATOM_BYTES = TILE * 128;           // 128 rows x 128 B
constexpr int S_BYTES = TILE * CHUNK * 2;        // 16 KB: one chunk of s
constexpr int W_BYTES = 16384;                   // one ring item
constexpr int NW = 4;
constexpr int kThreads = 608;
constexpr int TMEM_COLS = 512;

// kModeTile: the trunk transition (z tiles by TMA, LayerNorm in the kernel, fp16 residual).
// kModeH:    h = fp16(LN(z)) precomputed (a row LayerNorm pass), loaded by TMA straight into the
//            A-operand stages; t = fp16(D2) out.
enum Mode : int { kModeTile = 0, kModeH = 1 };

template <int CZ, int MODE = kModeTile>
struct Cfg {
  static constexpr int KATOMS = CZ / 64;
  static constexpr int TILE_BYTES = TILE * CZ * 2;                     // 32 or 64 KB
  static constexpr bool ROWS = MODE != kModeTile;                      // no z tile: h by TMA, t rows out
  static constexpr bool INPLACE = !ROWS && CZ == 256;                  // h overwrites z in its stage
  static constexpr int NACC = CZ == 128 ? 2 : 1;                       // D2 accumulators
  static constexpr int OFF_Z = 0;                                      // 2 stages (tile mode)
  static constexpr int OFF_H = (INPLACE || ROWS) ? OFF_Z : OFF_Z + 2 * TILE_BYTES;  // 2 stages
  static constexpr int OFF_S = OFF_H + 2 * TILE_BYTES;                 // 2 buffers
  static constexpr int OFF_W = OFF_S + 2 * S_BYTES;                    // NW ring items
  static constexpr int OFF_PAR = OFF_W + NW * W_BYTES;                 // fp32 LN gamma[c_z], beta[c_z]
  static constexpr int OFF_BAR = OFF_PAR + 2 * CZ * 4;
  static constexpr int SMEM_BYTES = OFF_BAR + 512;
  static_assert(SMEM_BYTES <= 232448, "K4 shared memory exceeds the per-block limit");
  static_assert(NACC * CZ + 2 * 128 <= TMEM_COLS, "K4 TMEM columns");
};

struct Params {
  CUtensorMap tm_z;    // z (kModeH: h) [B, L, L, c_z]: box {64, jw, ih, 1}, 128B swizzle (load)
  CUtensorMap tm_zo;   // z_out: box {64, min(jw,32), 32/min(jw,32), 1}, 128B swizzle (per-warp store)
  CUtensorMap tm_w12;  // w12 [W, c_z]: box {64, 64}, 128B swizzle
  CUtensorMap tm_w3;   // w3 [c_z, h]: box {64, 128}, 128B swizzle
  const __half* ln_w;
  const __half* ln_b;
  __half* tout;        // h mode: t = fp16(ffn(h)) [cells, c_z]
  int hidden;          // h
  int nchunk;          // h / 64
  int L, ih, jw, tiles_i, tiles_j, num_tiles;
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProdW = 0x401, kSiteProdZ = 0x402, kSiteLn = 0x403, kSiteMmaH = 0x404, kSiteMmaW = 0x405,
  kSiteMmaD1 = 0x406, kSiteMmaS = 0x407, kSiteMmaAcc = 0x408, kSiteAct = 0x409, kSiteEpi = 0x40a
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int per_b = p.tiles_i * p.tiles_j;
  bb = tile / per_b;
  const int r = tile - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <int CZ, bool SWIGLU, int MODE = kModeTile>
__global__ void __launch_bounds__(kThreads, 1) transition_kernel(const __grid_constant__ Params p) {
  const bool trace_on = trace_enabled(p.status);
  using C = Cfg<CZ, MODE>;
  constexpr uint32_t IDESC1 = idesc_f16_f32(128, 2 * CHUNK, false, false);
  constexpr uint32_t IDESC2 = idesc_f16_f32(128, 128, false, false);
  // Ring items per chunk.  GEMM1: one per 64-channel K atom, holding that atom of the chunk's
  // first 64 B rows and then of its next 64 (SwiGLU: x1 rows, x2 rows; ReLU: hidden units
  // 128k .. 128k+63, 128k+64 .. 128k+127): one N = 128 B operand.  GEMM2: one per 128 output
  // channels and s (NQ s per chunk).
  constexpr int G1_ITEMS = C::KATOMS;
  constexpr int G2_ITEMS = CZ / 128;
  constexpr int NQ = SWIGLU ? 1 : 2;
  extern __shared__ uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(p.status, kStatusLayout, 0x4ff);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* wfull = bars;           // [NW]
  uint64_t* wempty = bars + 4;      // [NW]
  uint64_t* zfull = bars + 8;       // [2]
  uint64_t* zempty = bars + 10;     // [2]
  uint64_t* hfull = bars + 12;      // [2]
  uint64_t* hempty = bars + 14;     // [2]
  uint64_t* d1full = bars + 16;     // [2]
  uint64_t* d1empty = bars + 18;    // [2]
  uint64_t* sfull = bars + 20;      // [2]
  uint64_t* sempty = bars + 22;     // [2]
  uint64_t* accfull = bars + 24;    // [2]
  uint64_t* accempty = bars + 26;   // [2]
  uint64_t& drain_bar = bars[28];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 29);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 29) + 4);
  volatile int* gflags = reinterpret_cast<volatile int*>(bars + 30);  // [4 groups][2] group_wait verdicts
  uint64_t* rfull = bars + 34;      // [2] c_z = 256: z reloaded for the epilogue
  // ReLU: GEMM2 of chunk c releases s buffer q on semptyq[2q + (c & 1)].  Every ReLU chunk uses
  // both s buffers, and the activation of chunk c may start while GEMM2 of chunk c - 2 still
  // runs, so one barrier per buffer would let its parity wait see a phase two back as done;
  // split by chunk parity, each barrier advances once per two chunks.
  uint64_t* semptyq = bars + 36;    // [4]
  float* par = reinterpret_cast<float*>(smem + C::OFF_PAR);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};
  const int n = p.nchunk;

  if (threadIdx.x == 0) {
    abort_sh = 0;
    for (int s = 0; s < NW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&zfull[s], 1);
      mbar_init(&zempty[s], 4);    // the four epilogue warps, after their stores read the tile
      mbar_init(&hfull[s], MODE == kModeH ? 1 : 4);  // the four LayerNorm warps, or the h loads
      mbar_init(&hempty[s], 1);    // the MMA, after the tile's last GEMM1
      mbar_init(&d1full[s], 1);
      mbar_init(&d1empty[s], 4);   // the four activation warps
      mbar_init(&sfull[s], 4);
      mbar_init(&sempty[s], 1);
      mbar_init(&accfull[s], 1);
      mbar_init(&accempty[s], 4);  // the four epilogue warps
      mbar_init(&rfull[s], 1);
    }
    for (int s = 0; s < 4; ++s) mbar_init(&semptyq[s], 1);
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  if (!C::ROWS)
    for (int i = threadIdx.x; i < 2 * CZ; i += blockDim.x) par[i] = __half2float(i < CZ ? p.ln_w[i] : p.ln_b[i - CZ]);
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_z);
    if (MODE == kModeTile) tma_prefetch_desc(&p.tm_zo);
    tma_prefetch_desc(&p.tm_w12);
    tma_prefetch_desc(&p.tm_w3);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  griddep_trigger();
  griddep_wait();
  trace_mark_start(p.status, trace_on);

  if (warp == 0) {
    // ---------------- weight ring producer, in the MMA's order: G1(j), then G2(j-2) ----------------
    if (lane == 0) {
      uint32_t r = 0;
      bool ok = true;
      // One ring item: two 64 x 64 boxes of w12 (at 0 and 8 KB), or one 64 x 128 box of w3.
      auto put = [&](const CUtensorMap* m, int c0, int c1, int c0b, int c1b, bool two) -> bool {
        const uint32_t s = r % NW, ph = (r / NW) & 1;
        if (!mbar_wait(&wempty[s], ph ^ 1, ctx, kSiteProdW)) return false;
        mbar_arrive_expect_tx(&wfull[s], W_BYTES);
        uint8_t* dst = smem + C::OFF_W + s * W_BYTES;
        tma_load_2d(dst, m, &wfull[s], c0, c1);
        if (two) tma_load_2d(dst + W_BYTES / 2, m, &wfull[s], c0b, c1b);
        ++r;
        return true;
      };
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        for (int j = 0; ok && j <= n + 1; ++j) {
          for (int k = 0; ok && j < n && k < G1_ITEMS; ++k) {  // w12 rows of chunk j
            if (SWIGLU)  // K atom k of the x1 rows over K atom k of the x2 rows
              ok = put(&p.tm_w12, k * 64, j * CHUNK, k * 64, p.hidden + j * CHUNK, true);
            else         // K atom k of rows 128j .. 128j+63 over rows 128j+64 .. (zero past h)
              ok = put(&p.tm_w12, k * 64, 2 * j * CHUNK, k * 64, (2 * j + 1) * CHUNK, true);
          }
          for (int q = 0; ok && j >= 2 && q < NQ; ++q)  // w3[128 m .. 128 m + 127, s q of chunk j-2]
            for (int m = 0; ok && m < G2_ITEMS; ++m) ok = put(&p.tm_w3, (NQ * (j - 2) + q) * CHUNK, m * 128, 0, 0, false);
        }
      }
      if (abort_sh) {  // drain the loads still in flight before the CTA exits
        for (uint32_t s = 0; s < NW; ++s) {
          const uint32_t armed = r > s ? (r - s + NW - 1) / NW : 0;
          if (armed) mbar_drain(&wfull[s], (armed - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 2) {
    // ---------------- h tile producer (kModeH): the stage is free after the tile's last GEMM1 ----------------
    if (lane == 0 && MODE == kModeH) {
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        if (!mbar_wait(&hempty[s], ph ^ 1, ctx, kSiteProdZ)) break;
        mbar_arrive_expect_tx(&hfull[s], C::TILE_BYTES);
        for (int a = 0; a < C::KATOMS; ++a)
          tma_load_4d(smem + C::OFF_H + s * C::TILE_BYTES + a * ATOM_BYTES, &p.tm_z, &hfull[s], a * 64, j0, i0, bb);
      }
      if (abort_sh) {
        for (uint32_t s = 0; s < 2; ++s) {
          const uint32_t armed = it > s ? (it - s + 1) / 2 : 0;
          if (armed) mbar_drain(&hfull[s], (armed - 1) & 1, 200000000ull);
        }
      }
    }
    // ---------------- z tile producer (tile mode) ----------------
    if (lane == 0 && MODE == kModeTile) {
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        if (!mbar_wait(&zempty[s], ph ^ 1, ctx, kSiteProdZ)) break;
        mbar_arrive_expect_tx(&zfull[s], C::TILE_BYTES);
        for (int a = 0; a < C::KATOMS; ++a)
          tma_load_4d(smem + C::OFF_Z + s * C::TILE_BYTES + a * ATOM_BYTES, &p.tm_z, &zfull[s], a * 64, j0, i0, bb);
      }
      if (abort_sh) {
        for (uint32_t s = 0; s < 2; ++s) {
          const uint32_t armed = it > s ? (it - s + 1) / 2 : 0;
          if (armed) mbar_drain(&zfull[s], (armed - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t r = 0, it = 0, gc = 0;  // ring item, tile, global chunk counters
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
        const uint32_t tb = it & 1, tph = (it >> 1) & 1;
        const uint32_t ab = it % C::NACC, aph = (it / C::NACC) & 1;
        if (!(ok = mbar_wait(&hfull[tb], tph, ctx, kSiteMmaH))) break;
        const uint64_t hdesc = sdesc_sw128(smem_u32(smem + C::OFF_H + tb * C::TILE_BYTES), 16, 1024);
        const uint32_t acc = tmem_base + ab * CZ;
        // GEMM1 runs two chunks ahead of GEMM2: G1(j) needs only that its TMEM buffer has been
        // read (by the activation of chunk j-2), so the tensor core computes chunk j while
        // chunks j-1 and j-2 are still being activated.
        for (int j = 0; ok && j <= n + 1; ++j) {
          if (j < n) {  // GEMM1 of chunk gc + j
            const uint32_t c = gc + j, b = c & 1, cph = (c >> 1) & 1;
            if (!(ok = mbar_wait(&d1empty[b], cph ^ 1, ctx, kSiteMmaD1))) break;
            const uint32_t d = tmem_base + 256 + b * 128;
            for (int k = 0; k < G1_ITEMS; ++k) {
              const uint32_t s = r % NW, ph = (r / NW) & 1;
              if (!(ok = mbar_wait(&wfull[s], ph, ctx, kSiteMmaW))) break;
              tc_fence_after();
              const uint64_t wdesc = sdesc_sw128(smem_u32(smem + C::OFF_W + s * W_BYTES), 16, 1024);
              // K atom k: D1[:, 0:64] = x1 (ReLU: the chunk's first 64), D1[:, 64:128] = x2 (its next 64)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_f16(d, sdesc_add(hdesc, k * ATOM_BYTES + kk * 32), sdesc_add(wdesc, kk * 32), IDESC1,
                         (k > 0 || kk > 0) ? 1u : 0u);
              umma_commit(&wempty[s]);
              ++r;
            }
            if (!ok) break;
            umma_commit(&d1full[b]);
            if (j == n - 1) umma_commit(&hempty[tb]);  // the tile's last read of h
          }
          if (j >= 2) {  // GEMM2 of chunk gc + j - 2
            const uint32_t c = gc + j - 2, b = c & 1, cph = (c >> 1) & 1;
            if (j == 2 && !(ok = mbar_wait(&accempty[ab], aph ^ 1, ctx, kSiteMmaAcc))) break;
            for (int q = 0; ok && q < NQ; ++q) {
              // SwiGLU: the chunk's s is in buffer c & 1; ReLU: its half q is in buffer q (every
              // chunk uses both)
              const uint32_t sb = SWIGLU ? b : q, sph = SWIGLU ? cph : (c & 1);
              if (!(ok = mbar_wait(&sfull[sb], sph, ctx, kSiteMmaS))) break;
              const uint64_t sdesc = sdesc_sw128(smem_u32(smem + C::OFF_S + sb * S_BYTES), 16, 1024);
              for (int m = 0; m < G2_ITEMS; ++m) {  // output channels [128 m, 128 m + 128)
                const uint32_t s = r % NW, ph = (r / NW) & 1;
                if (!(ok = mbar_wait(&wfull[s], ph, ctx, kSiteMmaW))) break;
                tc_fence_after();
                const uint64_t wdesc = sdesc_sw128(smem_u32(smem + C::OFF_W + s * W_BYTES), 16, 1024);
#pragma unroll
                for (int kk = 0; kk < CHUNK / 16; ++kk)
                  umma_f16(acc + m * 128, sdesc_add(sdesc, kk * 32), sdesc_add(wdesc, kk * 32), IDESC2,
                           (j > 2 || q > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&wempty[s]);
                ++r;
              }
              if (!ok) break;
              umma_commit(SWIGLU ? &sempty[sb] : &semptyq[2 * q + (c & 1)]);
            }
            if (!ok) break;
          }
        }
        if (!ok) break;
        umma_commit(&accfull[ab]);
        gc += n;
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < 7) {
    // ---------------- LayerNorm: z tile -> h ----------------
    const int row = threadIdx.x - 96;
    uint32_t it = 0, gcount = 0;
    if constexpr (MODE == kModeH) {
      // h arrives by TMA: nothing to normalise
    } else
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const uint32_t s = it & 1, ph = (it >> 1) & 1;
      if (C::INPLACE) {  // the stage is free once its z arrived (the previous tile there is done)
        if (!group_wait(&zfull[s], ph, nullptr, 0, ctx, kSiteLn, row == 0, 4, 128, gflags + 6, gcount)) break;
        uint8_t* X = smem + C::OFF_Z + s * C::TILE_BYTES;
        const float k = ln_row_shift(X, row);
        const float2 mr = ln256_moments(ln_half_sums(X, ATOM_BYTES, row, 0, k), ln_half_sums(X, ATOM_BYTES, row, 1, k),
                                        k, 1e-5f);
        ln_half_apply(X, X, ATOM_BYTES, row, 0, mr.x, mr.y, LnParSmem{par, par + CZ});
        ln_half_apply(X, X, ATOM_BYTES, row, 1, mr.x, mr.y, LnParSmem{par, par + CZ});
      } else {
        if (!group_wait(&hempty[s], ph ^ 1, &zfull[s], ph, ctx, kSiteLn, row == 0, 4, 128, gflags + 6, gcount)) break;
        ln_row128_sw128(smem + C::OFF_Z + s * C::TILE_BYTES, smem + C::OFF_H + s * C::TILE_BYTES, ATOM_BYTES, row,
                        1e-5f, LnParSmem{par, par + CZ});
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&hfull[s]);
    }
  } else if (warp < 15) {
    // ---------------- activation: D1 chunk -> s chunk (fp16, K-major swizzled) ----------------
    // Two groups of four warps; group g takes the chunks that use D1 / s buffer g (every other
    // chunk), so one group's TMEM-load latency hides behind the other's arithmetic.
    const int g = (warp - 7) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t tl = static_cast<uint32_t>(q * 32) << 16;
    const bool leader = (warp - 7) % 4 == 0 && lane == 0;
    uint32_t gc = 0, gcount = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
      for (int k = 0; k < n; ++k, ++gc) {
        if (static_cast<int>(gc & 1) != g) continue;
        const uint32_t b = g, cph = (gc >> 1) & 1;
        if (!(ok = group_wait(&d1full[b], cph, nullptr, 0, ctx, kSiteAct, leader, 1 + g, 128, gflags + 2 * g, gcount)))
          break;
        tc_fence_after();
        const uint32_t d = tmem_base + tl + 256 + b * 128;
        uint8_t* S = smem + C::OFF_S + b * S_BYTES;
        if (!SWIGLU) {
          // ReLU: the chunk's 128 hidden units in two halves of 64, half q into s buffer q.  Each
          // half is loaded and activated before waiting for its s buffer (GEMM2 of the previous
          // chunk done reading it), so the wait overlaps this warp's own work.
          for (int q = 0; q < 2; ++q) {
            uint32_t x[32], y[32];  // hidden units [64q, 64q + 32) and [64q + 32, 64q + 64) of the chunk
            tmem_ld32(d + 64 * q, x);
            tmem_ld32(d + 64 * q + 32, y);
            tmem_wait_ld2(x, y);
            if (q == 1) {  // the chunk buffer has been read: hand it back
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&d1empty[b]);
            }
            uint32_t o[32];
#pragma unroll
            for (int e = 0; e < 16; ++e) {  // relu(fp16(v)) == fp16(relu(v)): one rounding
              o[e] = pack_half2(fmaxf(__uint_as_float(x[2 * e]), 0.0f), fmaxf(__uint_as_float(x[2 * e + 1]), 0.0f));
              o[16 + e] = pack_half2(fmaxf(__uint_as_float(y[2 * e]), 0.0f), fmaxf(__uint_as_float(y[2 * e + 1]), 0.0f));
            }
            // buffer q is used by every chunk: wait for the previous chunk's GEMM2 of it (phase
            // (gc - 1) / 2 of its barrier for chunk parity (gc - 1) & 1)
            if (gc > 0 && !(ok = group_wait(&semptyq[2 * q + ((gc - 1) & 1)], ((gc - 1) >> 1) & 1, nullptr, 0, ctx,
                                            kSiteAct, leader, 1 + g, 128, gflags + 2 * g, gcount)))
              break;
            uint8_t* Sq = smem + C::OFF_S + q * S_BYTES;
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8)
              *reinterpret_cast<uint4*>(Sq + sw128_off(row, c8)) =
                  make_uint4(o[4 * c8], o[4 * c8 + 1], o[4 * c8 + 2], o[4 * c8 + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sfull[q]);
          }
          if (!ok) break;
        } else {
          // SwiGLU: the sigmoid makes this the longer computation; holding all 64 results would
          // spill, so wait for the s buffer first and store 16 hidden units at a time.
          if (!(ok = group_wait(&sempty[b], cph ^ 1, nullptr, 0, ctx, kSiteAct, leader, 1 + g, 128, gflags + 2 * g,
                                gcount)))
            break;
#pragma unroll 1
          for (int hq = 0; hq < 4; ++hq) {
            uint32_t x[16], y[16];
            tmem_ld16(d + hq * 16, x);
            tmem_ld16(d + CHUNK + hq * 16, y);
            tmem_wait_ld16x2(x, y);
            if (hq == 3) {  // the chunk buffer has been read: hand it back
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&d1empty[b]);
            }
            uint32_t o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              // a = fp16(x1), c = fp16(x2), sg = fp16(sigmoid(a)); the product of two fp16 values
              // is exact in fp32, so fp16(a * sg) and fp16(t * c) are single correctly rounded
              // fp16 multiplies, bit-identical to rounding the fp32 products
              const __half2 a = __floats2half2_rn(__uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1]));
              const __half2 c = __floats2half2_rn(__uint_as_float(y[2 * e]), __uint_as_float(y[2 * e + 1]));
              const float2 sf = sigmoid_f32x2(__half22float2(a));
              const __half2 r = __hmul2_rn(__hmul2_rn(a, __floats2half2_rn(sf.x, sf.y)), c);
              o[e] = *reinterpret_cast<const uint32_t*>(&r);
            }
            *reinterpret_cast<uint4*>(S + sw128_off(row, 2 * hq)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(S + sw128_off(row, 2 * hq + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sfull[b]);
        }
      }
    }
  } else {
    // ---------------- epilogue: z' = fp16(z + D2) over the z tile, per-warp TMA store ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int jo = (q * 32) % p.jw, io = (q * 32) / p.jw;  // this warp's 32 positions in the tile
    const uint32_t tl = static_cast<uint32_t>(q * 32) << 16;
    const bool leader = warp == 15 && lane == 0;
    uint32_t it = 0, gcount = 0;
    int reload_armed = -1;  // c_z = 256: the stage whose reload is in flight (for the abort drain)
    if constexpr (C::ROWS) {
      // h mode: t = fp16(D2), stored straight from registers.
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const uint32_t ab = it % C::NACC, aph = (it / C::NACC) & 1;
        if (!group_wait(&accfull[ab], aph, nullptr, 0, ctx, kSiteEpi, leader, 3, 128, gflags + 4, gcount)) break;
        tc_fence_after();
        const int gi = i0 + row / p.jw, gj = j0 + row % p.jw;
        const bool valid = gi < p.L && gj < p.L;
        uint4* dst = reinterpret_cast<uint4*>(p.tout + ((static_cast<size_t>(bb) * p.L + gi) * p.L + gj) * CZ);
#pragma unroll 1
        for (int c0 = 0; c0 < CZ; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tmem_base + tl + ab * CZ + c0, v);
          tmem_wait_ld(v);
          if (c0 + 32 == CZ) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accempty[ab]);
          }
          if (!valid) continue;
          uint32_t o[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = pack_half2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[c0 / 8 + e] = make_uint4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
        }
      }
    } else
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t tb = it & 1, tph = (it >> 1) & 1;
      const uint32_t ab = it % C::NACC, aph = (it / C::NACC) & 1;
      uint8_t* Z = smem + C::OFF_Z + tb * C::TILE_BYTES;
      if (C::INPLACE && leader && mbar_wait(&hempty[tb], tph, ctx, kSiteEpi)) {
        // The stage held h until the tile's last GEMM1: bring z back for the residual.
        mbar_arrive_expect_tx(&rfull[tb], C::TILE_BYTES);
        for (int a = 0; a < C::KATOMS; ++a) tma_load_4d(Z + a * ATOM_BYTES, &p.tm_z, &rfull[tb], a * 64, j0, i0, bb);
        reload_armed = static_cast<int>(tb);
      }
      if (!group_wait(&accfull[ab], aph, C::INPLACE ? &rfull[tb] : &zfull[tb], tph, ctx, kSiteEpi, leader, 3, 128,
                      gflags + 4, gcount))
        break;
      reload_armed = -1;
      tc_fence_after();
#pragma unroll 1
      for (int a = 0; a < C::KATOMS; ++a) {  // channels [64a, 64a + 64) = z atom a
        uint32_t v[32], u[32];
        tmem_ld32(tmem_base + tl + ab * CZ + a * 64, v);
        tmem_ld32(tmem_base + tl + ab * CZ + a * 64 + 32, u);
        tmem_wait_ld2(v, u);
        if (a == C::KATOMS - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[ab]);
        }
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {  // 8-channel chunks of the z row
          const uint32_t* acc = c8 < 4 ? v + 8 * c8 : u + 8 * (c8 - 4);
          uint8_t* zp = Z + a * ATOM_BYTES + sw128_off(row, c8);
          uint4 zv = *reinterpret_cast<const uint4*>(zp);
          uint32_t* zu = reinterpret_cast<uint32_t*>(&zv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 y = __fadd2_rn(unpack_half2(zu[e]),
                                        make_float2(__uint_as_float(acc[2 * e]), __uint_as_float(acc[2 * e + 1])));
            zu[e] = pack_half2(y.x, y.y);
          }
          *reinterpret_cast<uint4*>(zp) = zv;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        for (int a = 0; a < C::KATOMS; ++a)
          tma_store_4d(&p.tm_zo, Z + a * ATOM_BYTES + q * 32 * 128, a * 64, j0 + jo, i0 + io, bb);
        bulk_commit();
        bulk_wait_read<0>();
        mbar_arrive(&zempty[tb]);
      }
    }
    if (lane == 0) bulk_wait<0>();
    if (reload_armed >= 0) {  // an abort left a reload in flight: let it land before the CTA exits
      const uint32_t tb = static_cast<uint32_t>(reload_armed);
      mbar_drain(&rfull[tb], ((it >> 1) & 1), 200000000ull);
    }
  }

  tc_fence_before();
  __syncthreads();
  trace_mark_end(p.status, trace_on);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace k4
}  // namespace tmu
