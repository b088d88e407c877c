// K2: the triangle contraction as a persistent batched tcgen05 GEMM (fp16 in, fp32 TMEM
// accumulate, fp16 out).
//
// Reference: src/esmfold2_mlx/mlx_trunk.py:84-88 and mlx_trunk_kernels.py:219
//   outgoing  x[d,i,j] = sum_k a[d,i,k] * b[d,j,k]      (A = a[d],   B = b[d],   both K-major)
//   incoming  x[d,i,j] = sum_k a[d,k,i] * b[d,k,j]      (A = a[d]^T, B = b[d]^T, both MN-major)
// a, b, x live in HBM channel-major, one L x L matrix per (fold, channel) d, rows padded to a
// multiple of 8 elements (16-byte TMA strides); TMA zero-fills k >= L and clips stores at L.
//
// CTA = 6 warps: warp 0 issues TMA loads into a STAGES-deep ring, warp 1 allocates TMEM and
// one thread issues tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM accumulators, warps
// 2-5 drain the other accumulator (tcgen05.ld -> fp16 -> 128B-swizzled smem -> TMA store), so
// the epilogue of tile t overlaps the MMAs of tile t+1.  One CTA per SM, tiles strided over
// the grid, channel-major tile order so concurrent CTAs share a[d], b[d] in L2.
#pragma once

#include "tmu_common.cuh"

namespace tmu {
namespace k2 {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

// BN = 128, 192 or 256 columns per tile (the host picks the least padding for N: 192 serves
// 129-192 and 257-384, e.g. L = 146 and 384, where a 256-wide tile computes 43 % / 25 % padding)
template <int BN>
struct Cfg {
  static_assert(BN == 128 || BN == 192 || BN == 256, "K2 tile width");
  static constexpr int STAGES = (BN >= 192) ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STG_BYTES = BM * 64 * 2;  // one 64-column fp16 output chunk
  static constexpr int NSTG = 2;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + NSTG * STG_BYTES + 1024;  // + alignment slack
  static constexpr int TMEM_COLS = BN == 192 ? 512 : 2 * BN;  // two accumulators; allocations are powers of 2
};

struct Params {
  CUtensorMap tm_a;  // loads of a: K-major {K, M, Bc} box {64, 128, 1}, or MN-major box {64, 64, 1}
  CUtensorMap tm_b;  // loads of b: K-major {K, rows_per_part, Bc, parts} box {64, BN, 1, 1},
                     //             or MN-major box {64, 64, 1}
  CUtensorMap tm_x;  // store of x: {N, M, Bc}, box {64, 128, 1}, 128B swizzle
  int N;                 // columns of x = rows of the (possibly gathered) B operand
  int rows_per_part;     // K-major B: rows held by each part of a gathered buffer (BN divides it)
  int tiles_m, tiles_n, num_tiles, num_kb;
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int { kSiteProducer = 0x201, kSiteMmaTmem = 0x202, kSiteMmaFull = 0x203, kSiteEpilogue = 0x204 };

template <int BN, bool MN_MAJOR>
__global__ void __launch_bounds__(kThreads, 1) contract_kernel(const __grid_constant__ Params p) {
  const bool trace_on = trace_enabled(p.status);
  using C = Cfg<BN>;
  constexpr uint32_t IDESC = idesc_f16_f32(BM, BN, MN_MAJOR, MN_MAJOR);

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES], empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2], tempty_bar[2], drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  __shared__ volatile int ep_ok_sh;

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* stg = smem + C::STAGES * C::STAGE_BYTES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};

  if (threadIdx.x == 0) {
    abort_sh = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 128);
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_a);
    tma_prefetch_desc(&p.tm_b);
    tma_prefetch_desc(&p.tm_x);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  const int tiles_per_d = p.tiles_m * p.tiles_n;
  griddep_trigger();
  griddep_wait();  // a, b come from the previous kernel; x may still be read by it
  trace_mark_start(p.status, trace_on);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int d = tile / tiles_per_d;
        const int r = tile - d * tiles_per_d;
        const int m0 = (r / p.tiles_n) * BM;
        const int n0 = (r % p.tiles_n) * BN;
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const uint32_t s = it % C::STAGES, ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, ctx, kSiteProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          const int k0 = kb * BK;
          if (!MN_MAJOR) {
            tma_load_3d(sa, &p.tm_a, &full_bar[s], k0, m0, d);
            tma_load_4d(sb, &p.tm_b, &full_bar[s], k0, n0 % p.rows_per_part, d, n0 / p.rows_per_part);
          } else {
#pragma unroll
            for (int h = 0; h < BM / 64; ++h) tma_load_3d(sa + h * 8192, &p.tm_a, &full_bar[s], m0 + 64 * h, k0, d);
#pragma unroll
            for (int h = 0; h < BN / 64; ++h) tma_load_3d(sb + h * 8192, &p.tm_b, &full_bar[s], n0 + 64 * h, k0, d);
          }
        }
      }
      if (abort_sh) {  // wind down: let every armed load land before the CTA exits
        for (uint32_t s = 0; s < C::STAGES; ++s) {
          const uint32_t n_armed = it > s ? (it - s + C::STAGES - 1) / C::STAGES : 0;
          if (n_armed) mbar_drain(&full_bar[s], (n_armed - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++tcount) {
        const uint32_t acc = tcount & 1, aph = (tcount >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], aph ^ 1, ctx, kSiteMmaTmem)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dtm = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
          const uint32_t s = it % C::STAGES, ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, ctx, kSiteMmaFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t b_base = a_base + C::A_BYTES;
          // K-major: 16-element K steps 32 B apart (LBO unused); MN-major: 2 KB apart, 8 KB between
          // 64-wide M/N groups
          const uint64_t a0 = MN_MAJOR ? sdesc_sw128(a_base, 8192, 1024) : sdesc_sw128(a_base, 16, 1024);
          const uint64_t b0 = MN_MAJOR ? sdesc_sw128(b_base, 8192, 1024) : sdesc_sw128(b_base, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t step = MN_MAJOR ? kk * 2048 : kk * 32;
            umma_f16(dtm, sdesc_add(a0, step), sdesc_add(b0, step), IDESC, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty_bar[s]);  // the stage is free once these MMAs have read it
        }
        if (ok) umma_commit(&tfull_bar[acc]);
      }
      umma_commit(&drain_bar);  // completes once every MMA issued above has finished
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else {
    // ---------------- epilogue: TMEM -> fp16 -> swizzled smem -> TMA store ----------------
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = q * 32 + lane;
    const int ep = threadIdx.x - 64;
    uint32_t tcount = 0, stg_it = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++tcount) {
      const int d = tile / tiles_per_d;
      const int r = tile - d * tiles_per_d;
      const int m0 = (r / p.tiles_n) * BM;
      const int n0 = (r % p.tiles_n) * BN;
      const uint32_t acc = tcount & 1, aph = (tcount >> 1) & 1;
      // one thread waits (bounded) and the verdict is shared, so all 128 threads leave together
      if (ep == 0) ep_ok_sh = mbar_wait(&tfull_bar[acc], aph, ctx, kSiteEpilogue) ? 1 : 0;
      named_bar_sync(1, 128);
      if (!ep_ok_sh) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int ch = 0; ch < BN / 64; ++ch, ++stg_it) {
        uint32_t v0[32], v1[32];
        tmem_ld32(trow + ch * 64, v0);
        tmem_ld32(trow + ch * 64 + 32, v1);
        tmem_wait_ld2(v0, v1);
        if (ch == BN / 64 - 1) {
          tc_fence_before();
          mbar_arrive(&tempty_bar[acc]);  // accumulator fully read: MMA may reuse it
        }
        uint8_t* st = stg + (stg_it & 1) * C::STG_BYTES;
        if (ep == 0) bulk_wait_read<1>();  // the store that last used this buffer has read it
        named_bar_sync(1, 128);
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
          const uint32_t* v = (c16 < 4) ? (v0 + c16 * 8) : (v1 + (c16 - 4) * 8);
          uint4 o;
          o.x = pack_half2(__uint_as_float(v[0]), __uint_as_float(v[1]));
          o.y = pack_half2(__uint_as_float(v[2]), __uint_as_float(v[3]));
          o.z = pack_half2(__uint_as_float(v[4]), __uint_as_float(v[5]));
          o.w = pack_half2(__uint_as_float(v[6]), __uint_as_float(v[7]));
          *reinterpret_cast<uint4*>(st + sw128_off(row, c16)) = o;
        }
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (ep == 0) {
          if (n0 + ch * 64 < p.N) tma_store_3d(&p.tm_x, st, n0 + ch * 64, m0, d);
          bulk_commit();
        }
      }
    }
    if (ep == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  trace_mark_end(p.status, trace_on);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace k2
}  // namespace tmu
