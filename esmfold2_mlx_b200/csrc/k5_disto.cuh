// K5: the distogram head's expected distance per pair, the convergence signal of adaptive
// recycling (var_adaptive_loops.py:43-46,115-121):
//   logits[i,j] = (z[i,j] + z[j,i]) @ W^T + b            W [128 bins, c_z]
//   E[i,j]      = sum_k softmax(logits[i,j])_k * centre_k    (fp32)
// The symmetrised input is never formed: D = z_tile W^T + zT_tile W^T are two MMA chains into one
// TMEM accumulator, so the fp16 pair values enter the tensor core exactly.  The zT tile (element
// (i, j) = z[j, i]) comes from a second tensor map over the same z with the row and column
// strides swapped.  The softmax runs online over the 128 bins (32 at a time) in the epilogue.
//
// Tile = 128 positions (ih x jw block), M = 128 positions, N = 128 bins, K = 2 x c_z.
// CTA = 6 warps, persistent: warp 0 TMA (W once, then z and zT tiles, NSTAGE stages), warp 1
// TMEM (2 x 128 columns) + MMA, warps 2-5 epilogue (one TMEM lane quadrant = 32 positions each).
#pragma once

#include "tmu_common.cuh"

namespace tmu {
namespace k5 {

constexpr int TILE = 128;
constexpr int NBINS = 128;
constexpr int ATOM_BYTES = TILE * 128;  // 128 rows x 128 B (positions or bins)

template <int CZ>
struct Cfg {
  static constexpr int KATOMS = CZ / 64;
  static constexpr int W_BYTES = NBINS * CZ * 2;
  static constexpr int HALF_BYTES = TILE * CZ * 2;      // z or zT tile
  static constexpr int STAGE_BYTES = 2 * HALF_BYTES;
  static constexpr int NSTAGE = CZ == 128 ? 2 : 1;
  static constexpr int OFF_W = 0;
  static constexpr int OFF_Z = OFF_W + W_BYTES;
  static constexpr int OFF_PAR = OFF_Z + NSTAGE * STAGE_BYTES;  // fp32 bias[128], centres[128]
  static constexpr int OFF_BAR = OFF_PAR + 2 * NBINS * 4;
  static constexpr int SMEM_BYTES = OFF_BAR + 128;
  static_assert(SMEM_BYTES <= 232448, "K5 shared memory exceeds the per-block limit");
};

constexpr int kThreads = 192;
constexpr int TMEM_COLS = 256;

struct Params {
  CUtensorMap tm_z;   // z [B, L, L, c_z]: box {64, jw, ih, 1}
  CUtensorMap tm_zt;  // the same memory with row/column strides swapped (element (i, j) = z[j, i])
  CUtensorMap tm_w;   // W [128, c_z]: box {64, 128}
  const float* bias;     // [128] or null
  const float* centres;  // [128]
  float* out;            // E [B, L, L]
  int L, ih, jw, tiles_i, tiles_j, num_tiles;
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int { kSiteProd = 0x501, kSiteMmaW = 0x502, kSiteMmaZ = 0x503, kSiteMmaAcc = 0x504, kSiteEpi = 0x505 };

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int per_b = p.tiles_i * p.tiles_j;
  bb = tile / per_b;
  const int r = tile - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <int CZ>
__global__ void __launch_bounds__(kThreads, 1) disto_kernel(const __grid_constant__ Params p) {
  using C = Cfg<CZ>;
  constexpr uint32_t IDESC = idesc_f16_f32(128, NBINS, false, false);
  extern __shared__ uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(p.status, kStatusLayout, 0x5ff);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t& w_bar = bars[0];
  uint64_t* zfull = bars + 1;     // [NSTAGE]
  uint64_t* zempty = bars + 3;    // [NSTAGE]
  uint64_t* accfull = bars + 5;   // [2]
  uint64_t* accempty = bars + 7;  // [2]
  uint64_t& drain_bar = bars[9];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 10);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 10) + 4);
  volatile int* gflags = reinterpret_cast<volatile int*>(bars + 11);  // [2] group_wait verdicts
  float* bias = reinterpret_cast<float*>(smem + C::OFF_PAR);
  float* centres = bias + NBINS;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&w_bar, 1);
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(&zfull[s], 1);
      mbar_init(&zempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&accfull[s], 1);
      mbar_init(&accempty[s], 4);
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < NBINS; i += blockDim.x) {
    bias[i] = p.bias ? p.bias[i] : 0.0f;
    centres[i] = p.centres[i];
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_z);
    tma_prefetch_desc(&p.tm_zt);
    tma_prefetch_desc(&p.tm_w);
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
    mbar_arrive_expect_tx(&w_bar, C::W_BYTES);
    for (int a = 0; a < C::KATOMS; ++a) tma_load_2d(smem + C::OFF_W + a * ATOM_BYTES, &p.tm_w, &w_bar, a * 64, 0);
  }
  griddep_trigger();
  griddep_wait();

  if (warp == 0) {
    // ---------------- TMA producer: z and zT tiles ----------------
    if (lane == 0) {
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const uint32_t s = it % C::NSTAGE, ph = (it / C::NSTAGE) & 1;
        if (!mbar_wait(&zempty[s], ph ^ 1, ctx, kSiteProd)) break;
        mbar_arrive_expect_tx(&zfull[s], C::STAGE_BYTES);
        uint8_t* st = smem + C::OFF_Z + s * C::STAGE_BYTES;
        for (int a = 0; a < C::KATOMS; ++a) {
          tma_load_4d(st + a * ATOM_BYTES, &p.tm_z, &zfull[s], a * 64, j0, i0, bb);
          tma_load_4d(st + C::HALF_BYTES + a * ATOM_BYTES, &p.tm_zt, &zfull[s], a * 64, j0, i0, bb);
        }
      }
      if (abort_sh) {
        mbar_drain(&w_bar, 0, 200000000ull);
        for (uint32_t s = 0; s < static_cast<uint32_t>(C::NSTAGE); ++s) {
          const uint32_t armed = it > s ? (it - s + C::NSTAGE - 1) / C::NSTAGE : 0;
          if (armed) mbar_drain(&zfull[s], (armed - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA: D = z W^T + zT W^T ----------------
    if (lane == 0) {
      bool ok = mbar_wait(&w_bar, 0, ctx, kSiteMmaW);
      const uint32_t wb = smem_u32(smem + C::OFF_W);
      uint32_t it = 0;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++it) {
        const uint32_t s = it % C::NSTAGE, ph = (it / C::NSTAGE) & 1;
        const uint32_t b = it & 1, bph = (it >> 1) & 1;
        if (!(ok = mbar_wait(&zfull[s], ph, ctx, kSiteMmaZ))) break;
        if (!(ok = mbar_wait(&accempty[b], bph ^ 1, ctx, kSiteMmaAcc))) break;
        tc_fence_after();
        const uint64_t zd = sdesc_sw128(smem_u32(smem + C::OFF_Z + s * C::STAGE_BYTES), 16, 1024);
        const uint64_t wd = sdesc_sw128(wb, 16, 1024);
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int kk = 0; kk < CZ / 16; ++kk) {
            const uint32_t off = (kk >> 2) * ATOM_BYTES + (kk & 3) * 32;
            umma_f16(tmem_base + b * NBINS, sdesc_add(zd, half * C::HALF_BYTES + off), sdesc_add(wd, off), IDESC,
                     (half > 0 || kk > 0) ? 1u : 0u);
          }
        umma_commit(&zempty[s]);
        umma_commit(&accfull[b]);
      }
      umma_commit(&drain_bar);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else {
    // ---------------- epilogue: online softmax over the bins, expected distance ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;  // tile position
    const uint32_t tl = static_cast<uint32_t>(q * 32) << 16;
    constexpr float kLog2e = 1.4426950408889634f;
    uint32_t it = 0, gcount = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t b = it & 1, bph = (it >> 1) & 1;
      if (!group_wait(&accfull[b], bph, nullptr, 0, ctx, kSiteEpi, warp == 2 && lane == 0, 1, 128, gflags, gcount))
        break;
      tc_fence_after();
      float m = -INFINITY, den = 0.0f, num = 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < NBINS; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem_base + tl + b * NBINS + c0, v);
        tmem_wait_ld(v);
        if (c0 == NBINS - 32) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[b]);
        }
        float l[32];
        float cm = m;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          l[k] = (__uint_as_float(v[k]) + bias[c0 + k]) * kLog2e;  // logits in log2 units
          cm = fmaxf(cm, l[k]);
        }
        const float scale = ex2_approx(m - cm);  // rescale the running sums to the new maximum
        den *= scale;
        num *= scale;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float e = ex2_approx(l[k] - cm);
          den += e;
          num = fmaf(e, centres[c0 + k], num);
        }
        m = cm;
      }
      const int gi = i0 + row / p.jw, gj = j0 + row % p.jw;
      if (gi < p.L && gj < p.L) p.out[(static_cast<size_t>(bb) * p.L + gi) * p.L + gj] = num / den;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace k5
}  // namespace tmu
