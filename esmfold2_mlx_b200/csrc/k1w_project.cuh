// K1W: K1 for c_z = c = 256, the pair width of ESMFold2's released trunk (mlx_trunk.py:4).
// Same arithmetic as K1 (mlx_trunk.py:72-76,81-83; mlx_trunk_kernels.py:47-80,214-216):
//   n = fp16(LN(z)), proj = fp16(n @ w_in [+ b]), a/b = fp16(signal * sigmoid(gate) * mask).
//
// Why a separate kernel: the packed projection weights are 4c x c_z fp16 = 512 KB, more than an
// SM's shared memory, so they cannot all stay resident as in K1.  Instead the output is split
// into four weight sets -- {a, b} x {channels 0-127, 128-255}, each its 128 signal rows and 128
// gate rows (128 KB) -- and every CTA keeps ONE set resident for its whole life.  Tile t is
// (set t mod 4, position tile t / 4) and the grid is a multiple of 4, so a CTA's set never
// changes, and the four CTAs that need the same z tile work on it at the same time (the second
// to fourth read hits L2).  The cost is that each position's LayerNorm is computed four times.
//
// One tile = 64 pair positions (an ih x jw block, ih * jw = 64); D = W n^T with M = 128 output
// channels, N = 64 positions, K = 256 (signal rows into TMEM columns [0, 64) of a slot, gate
// rows into [64, 128)).  CTA = 22 warps, one per SM, persistent:
//   warp 0      TMA: this CTA's weight set once, then z tiles (2 stages of 32 KB, 128B swizzle)
//   warp 1      TMEM (4 slots x 128 columns; tile t uses slot t mod 4) and the MMA thread, whose
//               operand descriptors are built once per stage and advanced by constants
//   warps 2-5   LayerNorm in place: row = position, each row split over two warps (channel
//               halves) that exchange their partial sums through shared memory; + the mask
//   warps 6-21  epilogue: four groups of four warps (one per TMEM lane quadrant), group g drains
//               slot g; per 16 positions: gate, mask, fp16 into a 2 KB per-warp staging block,
//               and every 32 positions a TMA store of the 32-channel x 32-position box.
#pragma once

#include "tmu_common.cuh"

namespace tmu {
namespace k1w {

constexpr int CZ = 256;
constexpr int CC = 256;
constexpr int TILE = 64;
constexpr int KATOMS = CZ / 64;                  // 64-channel swizzle atoms along K
constexpr int ZATOM_BYTES = TILE * 128;          // 64 rows x 128 B
constexpr int WATOM_BYTES = 128 * 128;           // 128 weight rows x 128 B
constexpr int WBLOCK_BYTES = 128 * CZ * 2;       // 128 weight rows x 256 channels
constexpr int A_BYTES = TILE * CZ * 2;
constexpr int NSTAGE = 2;
constexpr int POS = 16;                          // positions per TMEM load
constexpr int SPOS = 32;                         // positions per TMA store
constexpr int WSTG_BYTES = 32 * SPOS * 2;
constexpr int NEPI = 16;
constexpr int NSLOT = 4;
constexpr int OFF_W = 0;                               // [signal rows | gate rows] of the set
constexpr int OFF_A = OFF_W + 2 * WBLOCK_BYTES;
constexpr int OFF_STG = OFF_A + NSTAGE * A_BYTES;
constexpr int OFF_PAR = OFF_STG + NEPI * WSTG_BYTES;   // fp16 LN gamma[256], beta[256]
constexpr int OFF_MASK = OFF_PAR + 2 * CZ * 2;         // fp16 mask [NSLOT][TILE]
constexpr int OFF_RED = OFF_MASK + NSLOT * TILE * 2;   // float2 [TILE]: LayerNorm half-row exchange
constexpr int OFF_BAR = OFF_RED + TILE * 8;
constexpr int SMEM_BYTES = OFF_BAR + 256;
constexpr int kThreads = 704;
constexpr int TMEM_COLS = 512;
static_assert(SMEM_BYTES <= 232448, "K1W shared memory exceeds the per-block limit");

struct Params {
  CUtensorMap tm_z;  // z [B, rows, cols, 256] (any element strides): box {64, jw, ih, 1}, 128B swizzle
  CUtensorMap tm_w;  // packed proj weights [1024, 256]: box {64, 128}, 128B swizzle
  CUtensorMap tm_a;  // a [B*256, rows, pitch]: box {min(jw,32), 32/min(jw,32), 32} (store)
  CUtensorMap tm_b;
  const __half* ln_w;
  const __half* ln_b;
  const float* bias;   // [4c] in packed-row order, or null
  const __half* mask;  // [B, rows, cols] with element strides mask_s*, or null
  long long mask_sb, mask_si, mask_sj;
  int rows, cols, ih, jw, log2_jw, tiles_i, tiles_j, num_tiles;  // num_tiles = 4 x position tiles
  int reset_status;
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProducer = 0x111, kSiteLn = 0x112, kSiteMmaW = 0x113, kSiteMmaLn = 0x114, kSiteMmaSlot = 0x115,
  kSiteEpilogue = 0x116
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int pt = tile >> 2;
  const int per_b = p.tiles_i * p.tiles_j;
  bb = pt / per_b;
  const int r = pt - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <bool HAS_BIAS, bool HAS_MASK>
__global__ void __launch_bounds__(kThreads, 1) project_gate_w_kernel(const __grid_constant__ Params p) {
  const bool trace_on = trace_enabled(p.status);
  constexpr uint32_t IDESC = idesc_f16_f32(128, 64, false, false);
  extern __shared__ uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(p.status, kStatusLayout, 0x11f);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t& w_bar = bars[0];
  uint64_t* zfull = bars + 1;
  uint64_t* zempty = bars + 3;
  uint64_t* lnfull = bars + 5;
  uint64_t* tfull = bars + 7;
  uint64_t* tempty = bars + 11;
  uint64_t* mfull = bars + 15;
  uint64_t* mempty = bars + 19;
  uint64_t& drain_bar = bars[23];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 24);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 24) + 4);
  volatile int& ln_ok_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 24) + 8);
  volatile int* gflags = reinterpret_cast<volatile int*>(bars + 26);  // [4 groups][2] group_wait verdicts
  __half* par = reinterpret_cast<__half*>(smem + OFF_PAR);     // [gamma 256 | beta 256]
  __half* maskh = reinterpret_cast<__half*>(smem + OFF_MASK);  // [NSLOT][64]
  float2* red = reinterpret_cast<float2*>(smem + OFF_RED);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};
  const int set = blockIdx.x & 3;            // constant: gridDim.x is a multiple of 4
  const int xsel = set >> 1, hsel = set & 1; // output a (0) or b (1); channel half

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
      mbar_init(&tempty[s], 4);  // the slot's four epilogue warps
      mbar_init(&mfull[s], 2);   // the two LayerNorm warps that write the mask
      mbar_init(&mempty[s], 4);
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 2 * CZ; i += blockDim.x) par[i] = i < CZ ? p.ln_w[i] : p.ln_b[i - CZ];
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
  if (warp == 0 && lane == 0) {  // weights are never written by this library: load before the wait
    mbar_arrive_expect_tx(&w_bar, 2 * WBLOCK_BYTES);
    for (int h = 0; h < 2; ++h) {
      const int row0 = (2 * xsel + h) * CC + hsel * 128;
      for (int a = 0; a < KATOMS; ++a)
        tma_load_2d(smem + OFF_W + h * WBLOCK_BYTES + a * WATOM_BYTES, &p.tm_w, &w_bar, a * 64, row0);
    }
  }
  griddep_trigger();
  griddep_wait();
  trace_mark_start(p.status, trace_on);
  // Block 0 clears (as in K1) this call's error fields once the previous kernel (which may share the word)
  // has finished.  Another CTA of this grid that gave up on a wait before block 0 got here
  // would have its per-call record cleared; its since-reset record (first_code) survives.
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
          tma_load_4d(smem + OFF_A + s * A_BYTES + a * ZATOM_BYTES, &p.tm_z, &zfull[s], a * 64, j0, i0, bb);
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
    // ---------------- MMA issuer: D[slot] = W n^T ----------------
    if (lane == 0) {
      bool ok = mbar_wait(&w_bar, 0, ctx, kSiteMmaW);
      uint32_t it = 0;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        const uint32_t slot = it & 3, sph = (it >> 2) & 1;
        if (!mbar_wait(&lnfull[s], ph, ctx, kSiteMmaLn)) break;
        if (!mbar_wait(&tempty[slot], sph ^ 1, ctx, kSiteMmaSlot)) break;
        tc_fence_after();
        const uint64_t n_desc = sdesc_sw128(smem_u32(smem + OFF_A + s * A_BYTES), 16, 1024);
        for (int h = 0; h < 2; ++h) {  // h = 0 signal rows, h = 1 gate rows
          const uint64_t w_desc = sdesc_sw128(smem_u32(smem + OFF_W + h * WBLOCK_BYTES), 16, 1024);
#pragma unroll
          for (int kk = 0; kk < CZ / 16; ++kk) {
            const uint32_t ka = (kk >> 2), kb = (kk & 3) * 32;
            umma_f16(tmem_base + slot * 128 + h * 64, sdesc_add(w_desc, ka * WATOM_BYTES + kb),
                     sdesc_add(n_desc, ka * ZATOM_BYTES + kb), IDESC, kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(&tfull[slot]);
        umma_commit(&zempty[s]);  // the n tile may be refilled once these MMAs have read it
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < 6) {
    // ---------------- LayerNorm in place (row split over two warps) + mask ----------------
    const int t = threadIdx.x - 64;
    const int row = t & 63, half = t >> 6;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const uint32_t s = it & 1, ph = (it >> 1) & 1;
      const uint32_t k = it & 3, mph = (it >> 2) & 1;
      // one thread waits (bounded) and shares the verdict, so all four warps always meet at the
      // named barriers below together
      if (t == 0) {
        bool ok = true;
        if (HAS_MASK) ok = mbar_wait(&mempty[k], mph ^ 1, ctx, kSiteLn);
        ok = ok && mbar_wait(&zfull[s], ph, ctx, kSiteLn);
        ln_ok_sh = ok ? 1 : 0;
      }
      named_bar_sync(1, 128);
      if (!ln_ok_sh) break;
      if (HAS_MASK && half == 0) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const int gi = i0 + row / p.jw, gj = j0 + row % p.jw;
        __half m = __float2half(0.0f);
        if (gi < p.rows && gj < p.cols) m = p.mask[bb * p.mask_sb + gi * p.mask_si + gj * p.mask_sj];
        maskh[k * TILE + row] = m;
        __syncwarp();
        if (lane == 0) mbar_arrive(&mfull[k]);
      }
      uint8_t* A = smem + OFF_A + s * A_BYTES;
      const float shift = ln_row_shift(A, row);
      const float2 sums = ln_half_sums(A, ZATOM_BYTES, row, half, shift);
      if (half) red[row] = sums;
      named_bar_sync(1, 128);
      if (!half) red[row] = ln256_moments(sums, red[row], shift, 1e-5f);
      named_bar_sync(1, 128);
      const float2 mr = red[row];
      ln_half_apply(A, A, ZATOM_BYTES, row, half, mr.x, mr.y, LnParSmemHalf{par, par + CZ});
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&lnfull[s]);
    }
  } else {
    // ---------------- epilogue: gate, mask, channel-major store ----------------
    const int g = (warp - 6) >> 2;  // slot drained by this group
    const int q = warp & 3;         // TMEM lane quadrant = channels [32q, 32q+32) of the half
    const int ch = q * 32 + lane;
    uint8_t* stg = smem + OFF_STG + (warp - 6) * WSTG_BYTES;
    uint32_t soff[2][2];
#pragma unroll
    for (int st = 0; st < 2; ++st)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (p.jw >= 32) {
          const uint32_t r = lane, cc = 2 * st + c;
          soff[st][c] = r * 64 + 16 * (cc ^ ((r >> 1) & 3));
        } else if (p.jw == 16) {
          const uint32_t r = 2 * lane + st;
          soff[st][c] = r * 32 + 16 * (c ^ ((r >> 2) & 1));
        } else {
          soff[st][c] = (4 * lane + 2 * st + c) * 16;
        }
      }
    float bs = 0.0f, bgt = 0.0f;
    if (HAS_BIAS) {
      bs = __ldg(p.bias + (2 * xsel) * CC + hsel * 128 + ch);
      bgt = __ldg(p.bias + (2 * xsel + 1) * CC + hsel * 128 + ch);
    }
    const float2 bs2 = make_float2(bs, bs), bg2 = make_float2(bgt, bgt);
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + g * 128;
    const CUtensorMap* tm = xsel == 0 ? &p.tm_a : &p.tm_b;
    const __half* mrow = maskh + g * TILE;
    uint32_t it = g, gcount = 0;
    const bool leader = ((warp - 6) & 3) == 0 && lane == 0;
    for (int tile = blockIdx.x + g * gridDim.x; tile < p.num_tiles; tile += 4 * gridDim.x, it += 4) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t sph = (it >> 2) & 1;
      // one thread of the group waits, the other warps park on barrier 2 + g
      if (!group_wait(&tfull[g], sph, HAS_MASK ? &mfull[g] : nullptr, sph, ctx, kSiteEpilogue, leader, 2 + g, 128,
                      gflags + 2 * g, gcount))
        break;
      tc_fence_after();
#pragma unroll 1
      for (int pb = 0; pb < TILE; pb += POS) {
        uint32_t sg[16], gt[16];
        tmem_ld16(taddr + pb, sg);
        tmem_ld16(taddr + 64 + pb, gt);
        tmem_wait_ld16x2(sg, gt);
        if (pb == TILE - POS) {  // the whole slot has been read: hand it back to the MMA
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[g]);
        }
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < POS; i += 2) {
          float2 sv = make_float2(__uint_as_float(sg[i]), __uint_as_float(sg[i + 1]));
          float2 gv = make_float2(__uint_as_float(gt[i]), __uint_as_float(gt[i + 1]));
          if (HAS_BIAS) {
            sv = __fadd2_rn(sv, bs2);
            gv = __fadd2_rn(gv, bg2);
          }
          sv = round_f16x2(sv);  // proj is an fp16 tensor in the reference
          gv = round_f16x2(gv);
          float2 y = __fmul2_rn(sv, sigmoid_f32x2(gv));
          if (HAS_MASK) y = __fmul2_rn(y, unpack_half2(*reinterpret_cast<const uint32_t*>(mrow + pb + i)));
          o[i / 2] = pack_half2(y.x, y.y);
        }
        const int step = (pb / POS) & 1;
        if (step == 0) {  // first half of a store box: the previous store must have read the block
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
        }
        const uint32_t off0 = step ? soff[1][0] : soff[0][0], off1 = step ? soff[1][1] : soff[0][1];
        *reinterpret_cast<uint4*>(stg + off0) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(stg + off1) = make_uint4(o[4], o[5], o[6], o[7]);
        if (step == 1) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int tp = pb - POS;  // tile position of the first of these 32
            tma_store_3d(tm, stg, j0 + (tp & (p.jw - 1)), i0 + (tp >> p.log2_jw), bb * CC + hsel * 128 + q * 32);
            bulk_commit();
          }
        }
      }
      if (HAS_MASK) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&mempty[g]);
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

}  // namespace k1w
}  // namespace tmu
