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
// The projection is computed transposed, D = W n^T (M = 128 output channels, N = 128 positions,
// K = c_z), so TMEM lane = channel and column = position: an epilogue thread owns one channel
// and reads 16 consecutive positions at a time, which are contiguous in the channel-major
// output.  Each of the four 128-row weight blocks (signal a, gate a, signal b, gate b) is one
// MMA chain over the whole tile into its own TMEM slot, so the tensor core reads every weight
// block once per tile (N = 64 chains over position halves read each twice, and the operand
// traffic through shared memory was the kernel's limiter); a signal and its gate share TMEM
// lanes, so they pair up in registers.
//
// One tile = 128 pair positions, an ih x jw block of the L x L grid (ih * jw = 128), chosen by
// the host by padded positions x a measured cost per position (wide tiles preferred from
// 512 x 512 positions up, the least padding below).  CTA = 26 warps, one per SM, persistent:
//   warp 0      TMA: packed weights once (resident, 4c x c_z fp16), then z tiles (2 stages)
//   warp 1      TMEM allocation (512 columns = 4 slots of 128 positions: signal a, gate a,
//               signal b, gate b) and the MMA thread, which refills the a (or b) slot pair as
//               soon as both epilogue groups of a (or b) have drained it
//   warps 2-9   LayerNorm of the z tile in place (a lane pair per position, each lane one half of
//               the channels, interleaved by 16-byte chunk) + the tile's mask as fp32
//   warps 10-25 epilogue: four groups {a, b} x {positions 0-63, 64-127} of four warps (one per
//               TMEM lane quadrant); per 16 positions:
//               gate, mask, fp16, 32 B per thread into a 2 KB staging block; every 32 positions
//               a per-warp TMA store of the 32-channel x 32-position box (64-byte rows when
//               jw >= 32), staged with the swizzle that keeps a warp's 32 row writes free of
//               bank conflicts.
#pragma once

#include "tmu_common.cuh"

namespace tmu {
namespace k1 {

constexpr int CZ = 128;  // c_z
constexpr int CC = 128;  // c (latent channels)
constexpr int TILE = 128;
constexpr int KATOMS = CZ / 64;              // 64-channel swizzle atoms along K
constexpr int ATOM_BYTES = TILE * 128;       // 128 rows x 128 B
constexpr int WBLOCK_BYTES = 128 * CZ * 2;   // 128 weight rows
constexpr int A_BYTES = TILE * CZ * 2;
constexpr int NSTAGE = 2;
constexpr int POS = 16;                      // positions per epilogue step (one TMEM load)
constexpr int SPOS = 32;                     // positions per TMA store (two steps)
constexpr int WSTG_BYTES = 32 * SPOS * 2;    // one warp's staging block (32 channels x 32 positions)
constexpr int NEPI = 16;
constexpr int NSLOT = 4;
constexpr int NMASK = 3;                     // mask stages (a tile's mask outlives its z stage)
constexpr int OFF_W = 0;                     // [sig_a | gate_a | sig_b | gate_b], 128 rows each
constexpr int OFF_A = OFF_W + 4 * WBLOCK_BYTES;
constexpr int OFF_STG = OFF_A + NSTAGE * A_BYTES;
constexpr int OFF_PAR = OFF_STG + NEPI * WSTG_BYTES;      // fp32 LN gamma, beta
constexpr int OFF_MASK = OFF_PAR + 2 * CZ * 4;            // fp32 mask per tile position
constexpr int OFF_BAR = OFF_MASK + NMASK * TILE * 4;     // mbarriers and flags
constexpr int SMEM_BYTES = OFF_BAR + 256;                 // no alignment slack: the kernel checks the base
constexpr int kThreads = 832;
constexpr int TMEM_COLS = 512;

struct Params {
  CUtensorMap tm_z;  // z [B, rows, cols, c_z] (any element strides): box {64, jw, ih, 1}, 128B swizzle
  CUtensorMap tm_w;  // packed proj weights [4c, c_z]: box {64, 128}, 128B swizzle
  CUtensorMap tm_a;  // a [B*c, L, Lpad]: box {min(jw,32), 32/min(jw,32), 32}, swizzle by jw (store)
  CUtensorMap tm_b;  // b, same
  const __half* ln_w;
  const __half* ln_b;
  const float* bias;   // [4c] in packed-row order, or null
  const __half* mask;  // [B, rows, cols] with element strides mask_s*, or null
  long long mask_sb, mask_si, mask_sj;
  int rows, cols, ih, jw, log2_jw, tiles_i, tiles_j, num_tiles;
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
  const bool trace_on = trace_enabled(p.status);
  constexpr uint32_t IDESC = idesc_f16_f32(128, 128, false, false);
  // All shared state lives in the dynamic buffer (no static __shared__), whose base the 128B
  // swizzle needs 1024-byte aligned; a misaligned base is reported, never computed on.
  extern __shared__ uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(p.status, kStatusLayout, 0x1ff);
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
  uint64_t* mempty = bars + 18;
  uint64_t& drain_bar = bars[21];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 22);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 22) + 4);
  volatile int* gflags = reinterpret_cast<volatile int*>(bars + 23);  // [5 groups][2] group_wait verdicts
  float* par = reinterpret_cast<float*>(smem + OFF_PAR);    // [gamma 128 | beta 128]
  float* maskf = reinterpret_cast<float*>(smem + OFF_MASK);  // [NMASK][128]
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&w_bar, 1);
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&zfull[s], 1);
      mbar_init(&zempty[s], 1);
      mbar_init(&lnfull[s], 8);  // one arrival per LayerNorm warp
    }
    for (int s = 0; s < NSLOT; ++s) {
      mbar_init(&tfull[s], 1);   // [0]: slots a, [1]: slots b
      mbar_init(&tempty[s], 8);  // the eight epilogue warps (two groups) draining a slot pair
    }
    for (int k = 0; k < NMASK; ++k) {
      mbar_init(&mfull[k], 8);      // LayerNorm warps wrote the tile's mask
      mbar_init(&mempty[k], NEPI);  // every epilogue warp is done with it
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  // Prologue (overlaps the previous kernel when launched with programmatic serialisation):
  // weights and parameters are never written by the kernels of this library, so they are
  // fetched before the dependency wait; z, mask, a, b and the status word only after it.
  for (int i = threadIdx.x; i < 2 * CZ; i += blockDim.x) par[i] = __half2float(i < CZ ? p.ln_w[i] : p.ln_b[i - CZ]);
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
    mbar_arrive_expect_tx(&w_bar, 4 * WBLOCK_BYTES);
    for (int q = 0; q < 4; ++q)
      for (int a = 0; a < KATOMS; ++a)
        tma_load_2d(smem + OFF_W + q * WBLOCK_BYTES + a * ATOM_BYTES, &p.tm_w, &w_bar, a * 64, q * 128);
  }
  griddep_trigger();
  griddep_wait();
  trace_mark_start(p.status, trace_on);
  // Block 0 clears this call's error fields once the previous kernel (which may share the word)
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
    // ---------------- MMA issuer: D[slot] = W_slot n^T ----------------
    if (lane == 0) {
      bool ok = mbar_wait(&w_bar, 0, ctx, kSiteMmaW);
      uint32_t it = 0;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
        const uint32_t s = it & 1, ph = (it >> 1) & 1;
        if (!mbar_wait(&lnfull[s], ph, ctx, kSiteMmaLn)) { ok = false; break; }
        tc_fence_after();
        const uint64_t n_desc = sdesc_sw128(smem_u32(smem + OFF_A + s * A_BYTES), 16, 1024);
        for (int x = 0; x < 2; ++x) {  // x = 0: a (slots 0, 1), x = 1: b (slots 2, 3)
          if (!mbar_wait(&tempty[x], (it & 1) ^ 1, ctx, kSiteMmaSlot)) { ok = false; break; }
          tc_fence_after();
          for (int h = 0; h < 2; ++h) {  // h = 0 signal rows, h = 1 gate rows: slot 2x + h
            const uint64_t w_desc = sdesc_sw128(smem_u32(smem + OFF_W + (2 * x + h) * WBLOCK_BYTES), 16, 1024);
#pragma unroll
            for (int kk = 0; kk < CZ / 16; ++kk) {
              const uint32_t off = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
              umma_f16(tmem_base + (2 * x + h) * 128, sdesc_add(w_desc, off), sdesc_add(n_desc, off), IDESC,
                       kk > 0 ? 1u : 0u);
            }
          }
          umma_commit(&tfull[x]);
        }
        if (ok) umma_commit(&zempty[s]);  // the z/n tile may be refilled once these MMAs have read it
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < 10) {
    // ---------------- LayerNorm of the z tile in place (a lane pair per row); the tile's mask ----------------
    const int row = (threadIdx.x - 64) >> 1, half = threadIdx.x & 1;
    uint32_t it = 0, gcount = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      const uint32_t s = it & 1, ph = (it >> 1) & 1;
      // one thread waits for the z tile (and the mask stage), the other warps park on barrier 1
      const uint32_t k = it % NMASK, mph = (it / NMASK) & 1;
      if (!group_wait(&zfull[s], ph, HAS_MASK ? &mempty[k] : nullptr, mph ^ 1, ctx, kSiteLn, threadIdx.x == 64, 1,
                      256, gflags, gcount))
        break;
      if (HAS_MASK) {  // stage k of the mask ring holds tiles k, k + NMASK, ...
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const int gi = i0 + row / p.jw, gj = j0 + row % p.jw;
        if (half == 0) {
          float m = 0.0f;
          if (gi < p.rows && gj < p.cols) m = __half2float(p.mask[bb * p.mask_sb + gi * p.mask_si + gj * p.mask_sj]);
          maskf[k * TILE + row] = m;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&mfull[k]);
      }
      uint8_t* A = smem + OFF_A + s * A_BYTES;
      // LayerNorm of the row by the lane pair, each lane's half (16-byte chunks c = 2i + half of
      // both atoms) read once into registers: shifted sums around the row's channel 0, one
      // shuffle to combine, then the normalised values written back in place.
      uint32_t u[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c16 = 2 * i + half;
        const uint4 v = *reinterpret_cast<const uint4*>(A + (c16 >> 3) * ATOM_BYTES + sw128_off(row, c16 & 7));
        u[4 * i] = v.x;
        u[4 * i + 1] = v.y;
        u[4 * i + 2] = v.z;
        u[4 * i + 3] = v.w;
      }
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
      const float rs = rsqrtf(var + 1e-5f);
      const float2 r2 = make_float2(rs, rs);
      const LnParSmem lpar{par, par + CZ};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c16 = 2 * i + half;
        float g[8], b[8];
        lpar(c16, g, b);
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          unsigned short lo, hi;
          split_half2(u[4 * i + e], lo, hi);
          const float2 d = __fmul2_rn(make_float2(add_f16_f32(lo, -mean), add_f16_f32(hi, -mean)), r2);
          const float2 y = __ffma2_rn(d, make_float2(g[2 * e], g[2 * e + 1]), make_float2(b[2 * e], b[2 * e + 1]));
          o[e] = pack_half2(y.x, y.y);
        }
        *reinterpret_cast<uint4*>(A + (c16 >> 3) * ATOM_BYTES + sw128_off(row, c16 & 7)) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
      __syncwarp();
      if (lane == 0) mbar_arrive(&lnfull[s]);
    }
  } else {
    // ---------------- epilogue: gate, mask, channel-major store ----------------
    const int grp = (warp - 10) >> 2;  // 2 * (a: 0, b: 1) + position half
    const int x = grp >> 1, hpos = grp & 1;
    const int q = warp & 3;            // TMEM lane quadrant = channels [32q, 32q+32)
    const int ch = q * 32 + lane;      // this thread's output channel
    uint8_t* stg = smem + OFF_STG + (warp - 10) * WSTG_BYTES;
    // Byte offsets in the staging block of this thread's two 16-byte chunks c of compute step
    // st (positions 16 st + 8 c ..), matching the store box and its swizzle:
    //   jw >= 32: box {32, 1, 32}, 64 B rows (row = channel), 64B swizzle
    //   jw == 16: box {16, 2, 32}, 32 B rows (row = 2 channel + st), 32B swizzle
    //   jw == 8:  box {8, 4, 32},  16 B rows (row = 4 channel + 2 st + c), no swizzle
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
    float bs = 0.0f, bg = 0.0f;
    if (HAS_BIAS) {
      bs = __ldg(p.bias + (2 * x) * 128 + ch);
      bg = __ldg(p.bias + (2 * x + 1) * 128 + ch);
    }
    const float2 bs2 = make_float2(bs, bs), bg2 = make_float2(bg, bg);
    // signal in slot 2x, gate in slot 2x + 1, this group's positions [64 hpos, 64 hpos + 64)
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + 2 * x * 128 + 64 * hpos;
    const CUtensorMap* tm = x == 0 ? &p.tm_a : &p.tm_b;
    uint32_t it = 0, gcount = 0;
    const bool leader = ((warp - 10) & 3) == 0 && lane == 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      // one thread of the group's four warps waits, the others park on barrier 2 + grp
      if (!group_wait(&tfull[x], it & 1, HAS_MASK ? &mfull[it % NMASK] : nullptr, (it / NMASK) & 1, ctx,
                      kSiteEpilogue, leader, 2 + grp, 128, gflags + 2 + 2 * grp, gcount))
        break;
      tc_fence_after();
      const float* mrow = maskf + (it % NMASK) * TILE + hpos * 64;
#pragma unroll 1
      for (int pb = 0; pb < 64; pb += POS) {
        uint32_t sg[16], gt[16];
        tmem_ld16(taddr + pb, sg);
        tmem_ld16(taddr + 128 + pb, gt);
        tmem_wait_ld16x2(sg, gt);
        if (pb == 64 - POS) {  // this group's part of the slot pair has been read
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[x]);
        }
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < POS; i += 2) {
          float2 s = make_float2(__uint_as_float(sg[i]), __uint_as_float(sg[i + 1]));
          float2 g = make_float2(__uint_as_float(gt[i]), __uint_as_float(gt[i + 1]));
          if (HAS_BIAS) {
            s = __fadd2_rn(s, bs2);
            g = __fadd2_rn(g, bg2);
          }
          s = round_f16x2(s);  // proj is an fp16 tensor in the reference
          g = round_f16x2(g);
          float2 y = __fmul2_rn(s, sigmoid_f32x2(g));
          if (HAS_MASK) y = __fmul2_rn(y, *reinterpret_cast<const float2*>(mrow + pb + i));
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
            const int tp = hpos * 64 + pb - POS;  // tile position of the first of these 32
            tma_store_3d(tm, stg, j0 + (tp & (p.jw - 1)), i0 + (tp >> p.log2_jw), bb * CC + q * 32);
            bulk_commit();
          }
        }
      }
      if (HAS_MASK) {  // this warp no longer reads the tile's mask
        __syncwarp();
        if (lane == 0) mbar_arrive(&mempty[it % NMASK]);
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

}  // namespace k1
}  // namespace tmu
