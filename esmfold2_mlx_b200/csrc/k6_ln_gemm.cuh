// K6: row LayerNorm followed by one projection, D = fp16(LN(x)) @ W^T, over the pair grid.  It
// serves the per-fold pair conditioning of the diffusion head (mlx_diffusion16.py:81-87, the
// pair16 precision of the adopted var_mlx_diffusion16 stack; f32 form mlx_diffusion.py:252-259):
//   stage A  z0   = fp16(fp16(LN(concat(z_trunk, rel_pos); z_input_norm)) @ z_proj)   [B,L,L,c]
//   stage D  bias = fp16(fp16(fp16(LN(z)) @ bias_w) + bias_b), stored as [nb, B, H, L, L]
// (bias_w / bias_b fold every token block's pair_norm affine into its pair_bias_proj:
// mlx_diffusion.py:85-89).
//
// Tile = 128 positions (ih x jw block); TMEM lane = position, column = output channel.
// CTA = 14 warps, one per SM, persistent:
//   warp 0      TMA: W streamed one 64-channel K atom (all N rows) per ring item, NW items
//   warp 1      TMEM (2 accumulators x N columns) + MMA thread: N = 16..256 in one instruction
//   warps 2-9   LayerNorm: one warp per row, coalesced loads from global memory, fp16 into
//               the swizzled A tile (HSTAGES tiles)
//   warps 10-13 epilogue: one TMEM lane quadrant (32 positions) each
// Every wait is bounded (status word + abort flag, as in the other kernels).
#pragma once

#include "ln_rows.cuh"

namespace tmu {
namespace k6 {

constexpr int TILE = 128;
constexpr int ATOM_BYTES = TILE * 128;
constexpr int NMAX = 256;
constexpr int NW = 3;
constexpr int kThreads = 448;
constexpr int TMEM_COLS = 512;

enum Epi : int { kEpiStore16 = 0, kEpiBiasT = 1 };

template <int K>
struct Cfg {
  static constexpr int NQ = K / 128;
  static constexpr int KATOMS = K / 64;
  static constexpr int H_BYTES = TILE * K * 2;
  static constexpr int HSTAGES = K <= 256 ? 2 : 1;
  static constexpr int RL = K <= 256 ? 4 : 2;  // rows each LayerNorm warp keeps in flight
  static constexpr int W_ITEM = NMAX * 128;  // one K atom of W for up to 256 output channels
  static constexpr int OFF_H = 0;
  static constexpr int OFF_W = HSTAGES * H_BYTES;
  static constexpr int OFF_BAR = OFF_W + NW * W_ITEM;
  static constexpr int SMEM_BYTES = OFF_BAR + 256;
  static_assert(SMEM_BYTES <= 232448, "K6 shared memory exceeds the per-block limit");
};

struct Params {
  CUtensorMap tm_w;       // W [N, K] fp16 (nn.Linear layout): box {64, N}, 128B swizzle
  const void* x1;         // row source (see RowSrc)
  const void* x2;
  int ld1, ld2;           // row pitch, elements
  const float* ln_g;      // [K] or null (no affine)
  const float* ln_b;
  void* out;              // kEpiStore16: fp16 [cells, N]; kEpiBiasT: fp16 [N / heads, B, heads, L, L]
  const __half* bias;     // [N] (kEpiBiasT)
  int n;                  // output channels N
  int heads;              // kEpiBiasT: H
  int B, L, ih, jw, tiles_i, tiles_j, num_tiles;
  float eps;
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProdW = 0x601, kSiteLn = 0x602, kSiteMmaH = 0x603, kSiteMmaAcc = 0x604, kSiteMmaW = 0x605, kSiteEpi = 0x606
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int per_b = p.tiles_i * p.tiles_j;
  bb = tile / per_b;
  const int r = tile - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <int K, int SRC, int EPI>
__global__ void __launch_bounds__(kThreads, 1) ln_gemm_kernel(const __grid_constant__ Params p) {
  using C = Cfg<K>;
  extern __shared__ uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0 && atomicCAS(&p.status->code, 0u, kStatusLayout) == 0u) p.status->site = 0x6ff;
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* wfull = bars;           // [NW]
  uint64_t* wempty = bars + 3;      // [NW]
  uint64_t* hfull = bars + 6;       // [2]
  uint64_t* hempty = bars + 8;      // [2]
  uint64_t* accfull = bars + 10;    // [2]
  uint64_t* accempty = bars + 12;   // [2]
  uint64_t& drain_bar = bars[14];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 15);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 15) + 4);
  volatile int* gflags = reinterpret_cast<volatile int*>(bars + 16);  // [2 groups][2] group_wait verdicts
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
    for (int s = 0; s < 2; ++s) {
      mbar_init(&hfull[s], 8);     // the eight LayerNorm warps
      mbar_init(&hempty[s], 1);    // the MMA, after the tile's GEMM
      mbar_init(&accfull[s], 1);
      mbar_init(&accempty[s], 4);  // the four epilogue warps
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&p.tm_w);
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
    // ---------------- W ring: K atom k of all N rows per item, every tile ----------------
    if (lane == 0) {
      uint32_t r = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        for (int k = 0; k < C::KATOMS; ++k, ++r) {
          const uint32_t s = r % NW, ph = (r / NW) & 1;
          if (!(ok = mbar_wait(&wempty[s], ph ^ 1, ctx, kSiteProdW))) break;
          mbar_arrive_expect_tx(&wfull[s], w_bytes);
          tma_load_2d(smem + C::OFF_W + s * C::W_ITEM, &p.tm_w, &wfull[s], k * 64, 0);
        }
      }
      if (abort_sh) {
        for (uint32_t s = 0; s < NW; ++s) {
          const uint32_t armed = r > s ? (r - s + NW - 1) / NW : 0;
          if (armed) mbar_drain(&wfull[s], (armed - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA: D[ab] = h W^T over the K atoms ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(128, p.n, false, false);
      uint32_t r = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
        const uint32_t hb = it % C::HSTAGES, hph = (it / C::HSTAGES) & 1;
        const uint32_t ab = it & 1, aph = (it >> 1) & 1;
        if (!(ok = mbar_wait(&hfull[hb], hph, ctx, kSiteMmaH))) break;
        if (!(ok = mbar_wait(&accempty[ab], aph ^ 1, ctx, kSiteMmaAcc))) break;
        const uint32_t hbase = smem_u32(smem + C::OFF_H + hb * C::H_BYTES);
        for (int k = 0; k < C::KATOMS; ++k, ++r) {
          const uint32_t s = r % NW, ph = (r / NW) & 1;
          if (!(ok = mbar_wait(&wfull[s], ph, ctx, kSiteMmaW))) break;
          tc_fence_after();
          const uint32_t wb = smem_u32(smem + C::OFF_W + s * C::W_ITEM);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem_base + ab * NMAX, sdesc_sw128(hbase + k * ATOM_BYTES + kk * 32, 16, 1024),
                     sdesc_sw128(wb + kk * 32, 16, 1024), idesc, (k > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&wempty[s]);
        }
        if (!ok) break;
        umma_commit(&hempty[hb]);
        umma_commit(&accfull[ab]);
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < 10) {
    // ---------------- LayerNorm: warp w normalises rows w, w + 8, .. of the tile ----------------
    const int w = warp - 2;
    float4 gg[C::NQ], bb4[C::NQ];
    const bool affine = p.ln_g != nullptr;
    load_ln_par<C::NQ>(p.ln_g, p.ln_b, lane, gg, bb4);
    uint32_t it = 0, gcount = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t hb = it % C::HSTAGES, hph = (it / C::HSTAGES) & 1;
      if (!group_wait(&hempty[hb], hph ^ 1, nullptr, 0, ctx, kSiteLn, warp == 2 && lane == 0, 1, 256, gflags, gcount))
        break;
      uint8_t* H = smem + C::OFF_H + hb * C::H_BYTES;
#pragma unroll 1
      for (int r0 = 0; r0 < 16; r0 += C::RL) {  // RL rows in flight per warp
        float4 v[C::RL][C::NQ];
        bool valid[C::RL];
#pragma unroll
        for (int u = 0; u < C::RL; ++u) {
          const int row = w + 8 * (r0 + u);
          const int gi = i0 + row / p.jw, gj = j0 + row % p.jw;
          valid[u] = gi < p.L && gj < p.L;
          if (valid[u])
            load_row<SRC, C::NQ>(p.x1, p.x2, (static_cast<size_t>(bb) * p.L + gi) * p.L + gj, p.ld1, p.ld2, lane,
                                 v[u]);
        }
#pragma unroll
        for (int u = 0; u < C::RL; ++u) {
          const int row = w + 8 * (r0 + u);
          if (valid[u])
            ln_row_store<C::NQ>(v[u], gg, bb4, affine, p.eps, H, ATOM_BYTES, row, lane);
          else
            zero_row_store<C::NQ>(H, ATOM_BYTES, row, lane);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&hfull[hb]);
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t tl = static_cast<uint32_t>(q * 32) << 16;
    uint32_t it = 0, gcount = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t ab = it & 1, aph = (it >> 1) & 1;
      if (!group_wait(&accfull[ab], aph, nullptr, 0, ctx, kSiteEpi, warp == 10 && lane == 0, 2, 128, gflags + 2,
                      gcount))
        break;
      tc_fence_after();
      const int gi = i0 + row / p.jw, gj = j0 + row % p.jw;
      const bool valid = gi < p.L && gj < p.L;
      const size_t cell = (static_cast<size_t>(bb) * p.L + gi) * p.L + gj;
#pragma unroll 1
      for (int c0 = 0; c0 < p.n; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem_base + tl + ab * NMAX + c0, v);
        tmem_wait_ld16(v);
        if (c0 + 16 >= p.n) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[ab]);
        }
        if (!valid) continue;
        if (EPI == kEpiStore16) {
          uint32_t o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = pack_half2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + cell * p.n + c0);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        } else {  // fp16(fp16(D) + bias) at out[c / H, b, c % H, i, j]
          const size_t plane = static_cast<size_t>(p.L) * p.L;
          const size_t pos = static_cast<size_t>(gi) * p.L + gj;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int c = c0 + e;
            const float d = round_f16(__uint_as_float(v[e]));
            const float y = d + __half2float(p.bias[c]);
            const int blk = c / p.heads, hh = c - blk * p.heads;
            static_cast<__half*>(p.out)[((static_cast<size_t>(blk) * p.B + bb) * p.heads + hh) * plane + pos] =
                __float2half_rn(y);
          }
        }
      }
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
