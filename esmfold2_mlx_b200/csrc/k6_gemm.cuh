// K6: one projection D = h @ W^T over the pair grid, h = fp16(LN(x)) [B, L, L, K] produced by the
// row LayerNorm pass (lnr::ln_rows_kernel) and loaded by TMA.  It serves the per-fold pair
// conditioning of the diffusion head (mlx_diffusion16.py:81-87, the pair16 precision of the
// adopted var_mlx_diffusion16 stack; f32 form mlx_diffusion.py:252-259):
//   stage A  z0   = fp16(h @ z_proj^T),  h = fp16(LN(concat(z_trunk, rel_pos); z_input_norm))
//   stage D  bias = fp16(fp16(h @ bias_w^T) + bias_b), h = fp16(LN(z)) without affine, stored as
//            [nb, B, H, L, L]
// (bias_w / bias_b fold every token block's pair_norm affine into its pair_bias_proj:
// mlx_diffusion.py:85-89), and the parcae step of the 6B loop (var_6b_mlx_loop.py:67-71, fp32):
//   z' = a * z + LN(z_init + refined) @ B^T
// as an fp32-accurate bf16 GEMM: LN's output and B are each split into three bf16 parts
// (x = x0 + x1 + x2 to 24 bits) and the six products x_i B_j with i + j <= 2 are accumulated in
// fp32 TMEM, smallest first (truncation error ~2^-24 relative).  The K steps run from a
// schedule: step s multiplies A channels [a_coord[s], +64) by W columns [w_coord[s], +64).
//
// Tile = 128 positions (ih x jw block); TMEM lane = position, column = output channel.
// CTA = 12 warps, one per SM, persistent:
//   warp 0      TMA: W streamed one 64-channel K atom (all N rows) per ring item, NW items
//   warp 1      TMEM (2 accumulators x N columns) + MMA thread: N = 16..256 in one instruction
//   warp 2      TMA: h, one K atom of the tile per ring slot, NA slots
//   warp 3      idle
//   warps 4-11  epilogue: two warps per TMEM lane quadrant, each on half of the columns
// Every wait is bounded (status word + abort flag, as in the other kernels).
#pragma once

#include "ln_rows.cuh"

namespace tmu {
namespace k6 {

constexpr int TILE = 128;
constexpr int ATOM_BYTES = TILE * 128;
constexpr int NMAX = 256;
constexpr int NW = 3;   // W ring items (NMAX x 128 B each)
constexpr int NA = 7;   // A ring slots (one K atom each)
constexpr int kThreads = 384;
constexpr int TMEM_COLS = 512;
constexpr int OFF_A = 0;
constexpr int OFF_W = NA * ATOM_BYTES;
constexpr int OFF_PAR = OFF_W + NW * NMAX * 128;  // fp32 bias[NMAX], int64 plane offsets[NMAX]
constexpr int OFF_BAR = OFF_PAR + NMAX * 4 + NMAX * 8;
constexpr int SMEM_BYTES = OFF_BAR + 256;
static_assert(SMEM_BYTES <= 232448, "K6 shared memory exceeds the per-block limit");

enum Epi : int { kEpiStore16 = 0, kEpiBiasT = 1, kEpiAxpy = 2 };
constexpr int kMaxSteps = 32;

struct Params {
  CUtensorMap tm_w;       // W [N, K] fp16 (nn.Linear layout): box {64, N}, 128B swizzle
  CUtensorMap tm_a;       // h [B, L, L, K] fp16: box {64, jw, ih, 1}, 128B swizzle
  void* out;              // kEpiStore16: fp16 [cells, N]; kEpiBiasT: fp16 [N / heads, B, heads, L, L];
                          // kEpiAxpy: fp32 [cells, N]
  const __half* bias;     // [N] (kEpiBiasT)
  const float* zres;      // kEpiAxpy: z fp32 [cells, N] (may alias out)
  const float* avec;      // kEpiAxpy: a [N]
  int n;                  // output channels N
  int heads;              // kEpiBiasT: H
  int nsteps;             // K steps of 64 (<= kMaxSteps)
  short a_coord[kMaxSteps];
  short w_coord[kMaxSteps];
  int B, L, ih, jw, tiles_i, tiles_j, num_tiles;
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProdW = 0x601, kSiteProdA = 0x602, kSiteMmaA = 0x603, kSiteMmaAcc = 0x604, kSiteMmaW = 0x605, kSiteEpi = 0x606
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int per_b = p.tiles_i * p.tiles_j;
  bb = tile / per_b;
  const int r = tile - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <int EPI, bool BF16 = false>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ Params p) {
  const int nsteps = p.nsteps;
  extern __shared__ uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(p.status, kStatusLayout, 0x6ff);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* wfull = bars;            // [NW]
  uint64_t* wempty = bars + 3;       // [NW]
  uint64_t* afull = bars + 6;        // [NA]
  uint64_t* aempty = bars + 13;      // [NA]
  uint64_t* accfull = bars + 20;     // [2]
  uint64_t* accempty = bars + 22;    // [2]
  uint64_t& drain_bar = bars[24];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 25);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 25) + 4);
  volatile int* gflags = reinterpret_cast<volatile int*>(bars + 26);  // [2] group_wait verdicts
  float* bias_s = reinterpret_cast<float*>(smem + OFF_PAR);
  long long* plane_s = reinterpret_cast<long long*>(smem + OFF_PAR + NMAX * 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};
  const uint32_t w_bytes = static_cast<uint32_t>(p.n) * 128;

  if (threadIdx.x == 0) {
    abort_sh = 0;
    for (int s = 0; s < NW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int s = 0; s < NA; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&accfull[s], 1);
      mbar_init(&accempty[s], 8);  // the eight epilogue warps
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  if (EPI == kEpiAxpy)
    for (int c = threadIdx.x; c < p.n; c += blockDim.x) bias_s[c] = p.avec[c];
  if (EPI == kEpiBiasT) {
    // channel c = blk * H + hh lives in plane (blk * B + b) * H + hh of [nb, B, H, L, L]: the
    // b-independent part of its element offset, and its bias, once per CTA
    const long long plane = static_cast<long long>(p.L) * p.L;
    for (int c = threadIdx.x; c < p.n; c += blockDim.x) {
      const int blk = c / p.heads, hh = c - blk * p.heads;
      plane_s[c] = (static_cast<long long>(blk) * p.B * p.heads + hh) * plane;
      bias_s[c] = __half2float(p.bias[c]);
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_w);
    tma_prefetch_desc(&p.tm_a);
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

  if (warp == 0) {
    if (lane == 0) {  // W ring: K atom k of all N rows per item, every tile
      uint32_t r = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        for (int k = 0; k < nsteps; ++k, ++r) {
          const uint32_t s = r % NW, ph = (r / NW) & 1;
          if (!(ok = mbar_wait(&wempty[s], ph ^ 1, ctx, kSiteProdW))) break;
          mbar_arrive_expect_tx(&wfull[s], w_bytes);
          tma_load_2d(smem + OFF_W + s * NMAX * 128, &p.tm_w, &wfull[s], p.w_coord[k], 0);
        }
      }
      if (abort_sh) {
        for (uint32_t s = 0; s < NW; ++s) {
          const uint32_t armed = r > s ? (r - s + NW - 1) / NW : 0;
          if (armed) mbar_drain(&wfull[s], (armed - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {  // A ring: K atom k of the tile's h rows per slot
      uint32_t a = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        for (int k = 0; k < nsteps; ++k, ++a) {
          const uint32_t s = a % NA, ph = (a / NA) & 1;
          if (!(ok = mbar_wait(&aempty[s], ph ^ 1, ctx, kSiteProdA))) break;
          mbar_arrive_expect_tx(&afull[s], ATOM_BYTES);
          tma_load_4d(smem + OFF_A + s * ATOM_BYTES, &p.tm_a, &afull[s], p.a_coord[k], j0, i0, bb);
        }
      }
      if (abort_sh) {
        for (uint32_t s = 0; s < NA; ++s) {
          const uint32_t armed = a > s ? (a - s + NA - 1) / NA : 0;
          if (armed) mbar_drain(&afull[s], (armed - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = BF16 ? idesc_bf16_f32(128, p.n, false, false) : idesc_f16_f32(128, p.n, false, false);
      uint32_t r = 0, a = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
        const uint32_t ab = it & 1, aph = (it >> 1) & 1;
        if (!(ok = mbar_wait(&accempty[ab], aph ^ 1, ctx, kSiteMmaAcc))) break;
        for (int k = 0; k < nsteps; ++k, ++r, ++a) {
          const uint32_t sa = a % NA, sw = r % NW;
          if (!(ok = mbar_wait(&afull[sa], (a / NA) & 1, ctx, kSiteMmaA))) break;
          if (!(ok = mbar_wait(&wfull[sw], (r / NW) & 1, ctx, kSiteMmaW))) break;
          tc_fence_after();
          const uint64_t had = sdesc_sw128(smem_u32(smem + OFF_A + sa * ATOM_BYTES), 16, 1024);
          const uint64_t wbd = sdesc_sw128(smem_u32(smem + OFF_W + sw * NMAX * 128), 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem_base + ab * NMAX, sdesc_add(had, kk * 32), sdesc_add(wbd, kk * 32), idesc,
                     (k > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&aempty[sa]);
          umma_commit(&wempty[sw]);
        }
        if (!ok) break;
        umma_commit(&accfull[ab]);
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp >= 4) {
    // ---------------- epilogue: warp (q, e) takes TMEM quadrant q, column half e ----------------
    const int q = warp & 3;
    const int e = (warp - 4) >> 2;
    const int row = q * 32 + lane;
    const uint32_t tl = static_cast<uint32_t>(q * 32) << 16;
    const bool split = p.n % 32 == 0;
    const int ncol = split ? p.n / 2 : (e == 0 ? p.n : 0);
    const int cbeg = split ? e * ncol : 0;
    uint32_t it = 0, gcount = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t ab = it & 1, aph = (it >> 1) & 1;
      if (!group_wait(&accfull[ab], aph, nullptr, 0, ctx, kSiteEpi, warp == 4 && lane == 0, 2, 256, gflags, gcount))
        break;
      tc_fence_after();
      const int gi = i0 + row / p.jw, gj = j0 + row % p.jw;
      const bool valid = gi < p.L && gj < p.L;
      const size_t cell = (static_cast<size_t>(bb) * p.L + gi) * p.L + gj;
      const long long pos = static_cast<long long>(bb) * p.heads * p.L * p.L + static_cast<long long>(gi) * p.L + gj;
#pragma unroll 1
      for (int c0 = cbeg; c0 < cbeg + ncol; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem_base + tl + ab * NMAX + c0, v);
        tmem_wait_ld16(v);
        if (!valid) continue;
        if (EPI == kEpiStore16) {
          uint32_t o[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] = pack_half2(__uint_as_float(v[2 * k]), __uint_as_float(v[2 * k + 1]));
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + cell * p.n + c0);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        } else if (EPI == kEpiBiasT) {  // fp16(fp16(D) + bias) at out[c / H, b, c % H, i, j]
          __half* out = static_cast<__half*>(p.out) + pos;
#pragma unroll
          for (int k = 0; k < 16; ++k)
            out[plane_s[c0 + k]] = __float2half_rn(round_f16(__uint_as_float(v[k])) + bias_s[c0 + k]);
        } else {  // a * z + D, fp32 (z read before its row is written: same thread, same columns)
          const float4* zr = reinterpret_cast<const float4*>(p.zres + cell * p.n + c0);
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + cell * p.n + c0);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 z = zr[k];
            const float* av = bias_s + c0 + 4 * k;
            dst[k] = make_float4(fmaf(av[0], z.x, __uint_as_float(v[4 * k])), fmaf(av[1], z.y, __uint_as_float(v[4 * k + 1])),
                                 fmaf(av[2], z.z, __uint_as_float(v[4 * k + 2])),
                                 fmaf(av[3], z.w, __uint_as_float(v[4 * k + 3])));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace k6
}  // namespace tmu
