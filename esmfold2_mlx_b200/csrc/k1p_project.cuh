// K1P: K1 on CTA pairs, for c_z = c = 128 and 256.  Same arithmetic as K1 (mlx_trunk.py:72-76,
// 81-83; mlx_trunk_kernels.py:47-80,214-216):
//   n = fp16(LN(z)), proj = fp16(n @ w_in [+ b]), a/b = fp16(signal * sigmoid(gate) * mask).
//
// A cluster of two CTAs on two SMs projects a tile of 128 positions through MMAs that span both
// SMs (tcgen05 .cta_group::2, M = 256 output rows, N = 128 positions, K = c_z).  CTA r holds the
// A operand's rows [128 r, 128 r + 128) of two MMA chains (signal, gate) resident, normalises ITS
// 64 of the tile's 128 positions (the B operand's half), and receives in its TMEM the signal and
// gate projections of its 128 output channels for all 128 positions, so an epilogue thread has a
// channel's signal and gate side by side:
//   c_z = 256: the packed weights are 4c x c_z fp16 = 512 KB, so a pair computes one operand (a
//              or b: signal chain = its 256 signal rows, gate chain = its 256 gate rows; CTA r
//              takes channels [128 r, 128 r + 128)).  Pairs alternate between the operands (the
//              pair count is even): every LayerNorm is computed twice, once per operand.
//   c_z = 128: a pair computes both operands (signal chain = [signal a; signal b], gate chain
//              = [gate a; gate b]: CTA 0 produces a, CTA 1 produces b) from 64 KB of weights per
//              CTA, which leaves room for four z stages; every LayerNorm is computed once.
// One MMA instruction covers 256 x 128 outputs (the single-CTA K1: 128 x 128), and the two TMEM
// slots double-buffer the accumulators (the single-CTA K1 fills all of TMEM with one tile).
// The library launches the c_z = 256 form.  The c_z = 128 form passes the same parity tests but
// measured slower than the single-CTA K1 (L = 1024: 309 vs 219 us; L = 238: 26.0 vs 24.2 us), so
// K1 keeps c_z = 128.
//
// Tile = 128 positions as an ih x jw block (ih * jw = 128); CTA r's piece is rows
// [ih/2 r, ih/2 r + ih/2) of it (ih >= 2) or columns [64 r, 64 r + 64) (ih = 1), so the
// accumulator's columns are the tile's positions in row-major order.  Per CTA, 26 warps:
//   warp 0      TMA: the weight halves once; per tile its piece of z (64 positions x c_z
//               channels, [c_z/64 atoms][64 rows][128 B], 128B swizzle), NSTAGE stages
//   warp 1      TMEM (2 slots x 256 columns: signal [0, 128), gate [128, 256), allocated for the
//               pair) and, in the even CTA, the MMA thread
//   warps 2-9   LayerNorm of the piece in place: a row on four adjacent lanes, lane k holding the
//               row's 16-byte chunks k and k + 4 of every atom (odd rows take them in the other
//               order, so the eight lanes of a shared-memory phase hit eight bank groups),
//               combined by two shuffles; plus the tile's mask (all 128 positions)
//   warps 10-25 epilogue: four groups of four warps (one per TMEM lane quadrant), group g takes
//               positions [32 g, 32 g + 32): gate, mask, fp16 into a 2 KB staging block, one
//               TMA store of the 32-channel x 32-position box.
// Cross-CTA traffic is mbarrier signals only (operand-ready and accumulator-free arrivals on the
// even CTA's barriers, multicast commits to both).
#pragma once

#include "tmu_common.cuh"

namespace tmu {
namespace k1p {

constexpr int TILE = 128;                        // positions per pair tile
constexpr int PT = 64;                           // positions per CTA
constexpr int ZATOM_BYTES = PT * 128;            // 64 rows x 128 B
constexpr int WATOM_BYTES = 128 * 128;           // 128 weight rows x 128 B
constexpr int POS = 16;                          // positions per TMEM load
constexpr int SPOS = 32;                         // positions per TMA store
constexpr int WSTG_BYTES = 32 * SPOS * 2;
constexpr int NEPI = 16;
constexpr int NMASK = 3;                         // mask ring (a tile's mask outlives its z stage)
constexpr int kThreads = 832;
constexpr int EPI_WARP0 = 10;
constexpr int TMEM_COLS = 512;

template <int CZ>
struct Cfg {
  static constexpr int KATOMS = CZ / 64;                  // 64-channel swizzle atoms along K
  static constexpr int WBLOCK_BYTES = 128 * CZ * 2;       // 128 weight rows x c_z channels
  static constexpr int PIECE_BYTES = PT * CZ * 2;         // 64 positions x c_z channels
  static constexpr int NSTAGE = CZ == 256 ? 2 : 4;        // z stages beside the resident weights
  static constexpr int OFF_W = 0;                         // [signal rows | gate rows]
  static constexpr int OFF_A = OFF_W + 2 * WBLOCK_BYTES;  // NSTAGE stages: the z piece, then n in place
  static constexpr int OFF_STG = OFF_A + NSTAGE * PIECE_BYTES;
  static constexpr int OFF_PAR = OFF_STG + NEPI * WSTG_BYTES;  // fp16 LN gamma[c_z], beta[c_z]
  static constexpr int OFF_MASK = OFF_PAR + 2 * CZ * 2;        // fp16 mask [NMASK][TILE]
  static constexpr int OFF_BAR = OFF_MASK + NMASK * TILE * 2;
  static constexpr int SMEM_BYTES = OFF_BAR + 256;
  static_assert(SMEM_BYTES <= 232448, "K1P shared memory exceeds the per-block limit");
};

struct Params {
  CUtensorMap tm_z;  // z [B, rows, cols, c_z] (any element strides): box {64, piece cols, piece rows, 1}, 128B swizzle
  CUtensorMap tm_w;  // packed proj weights [4 c, c_z]: box {64, 128}, 128B swizzle
  CUtensorMap tm_a;  // a [B*c, rows, pitch]: box {min(jw,32), 32/min(jw,32), 32} (store)
  CUtensorMap tm_b;
  const __half* ln_w;
  const __half* ln_b;
  const float* bias;   // [4c] in packed-row order, or null
  const __half* mask;  // [B, rows, cols] with element strides mask_s*, or null
  long long mask_sb, mask_si, mask_sj;
  int rows, cols, ih, jw, log2_jw, tiles_i, tiles_j, num_tiles;  // c_z = 256: num_tiles = 2 x position tiles
  int reset_status;
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProducer = 0x131, kSiteLn = 0x132, kSiteMmaW = 0x133, kSiteMmaLn = 0x134, kSiteMmaSlot = 0x135,
  kSiteEpilogue = 0x136
};

template <int CZ>
__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int pt = CZ == 256 ? tile >> 1 : tile;  // c_z = 256: tile = (position tile, operand)
  const int per_b = p.tiles_i * p.tiles_j;
  bb = pt / per_b;
  const int r = pt - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <int CZ, bool HAS_BIAS, bool HAS_MASK>
__global__ void __launch_bounds__(kThreads, 1) project_gate_pair_kernel(const __grid_constant__ Params p) {
  using C = Cfg<CZ>;
  constexpr int CC = CZ;  // c == c_z
  constexpr int KATOMS = C::KATOMS, NSTAGE = C::NSTAGE, PIECE_BYTES = C::PIECE_BYTES, WBLOCK_BYTES = C::WBLOCK_BYTES;
  constexpr int OFF_W = C::OFF_W, OFF_A = C::OFF_A, OFF_STG = C::OFF_STG, OFF_PAR = C::OFF_PAR, OFF_MASK = C::OFF_MASK,
                OFF_BAR = C::OFF_BAR;
  const bool trace_on = trace_enabled(p.status);
  constexpr uint32_t IDESC = idesc_f16_f32(256, TILE, false, false);
  extern __shared__ uint8_t smem[];
  // Both CTAs of a cluster take the same branch (a property of the kernel), so neither can be
  // left waiting at the cluster barriers below.
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(p.status, kStatusLayout, 0x13f);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t& w_bar = bars[0];
  uint64_t& wpair = bars[1];     // even CTA: both weight halves resident (2 arrivals)
  uint64_t* zfull = bars + 2;    // [NSTAGE]
  uint64_t* zempty = bars + 6;   // [NSTAGE]: the paired MMAs have read n (multicast commit)
  uint64_t* lnfull = bars + 10;  // [NSTAGE], even CTA: both CTAs' LayerNorm warps (16 arrivals)
  uint64_t* tfull = bars + 14;   // [2 slots]: the accumulator slot is complete (multicast commit)
  uint64_t* tempty = bars + 16;  // [2 slots], even CTA: both CTAs' epilogue warps have read it (32 arrivals)
  uint64_t* mfull = bars + 18;   // [NMASK]: the LayerNorm warps wrote the tile's mask
  uint64_t* mempty = bars + 21;  // [NMASK]: every epilogue warp is done with it
  uint64_t& drain_bar = bars[24];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 25);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 25) + 4);
  volatile int* gflags = reinterpret_cast<volatile int*>(bars + 26);  // [5 groups][2] group_wait verdicts
  __half* par = reinterpret_cast<__half*>(smem + OFF_PAR);     // [gamma c_z | beta c_z]
  __half* maskh = reinterpret_cast<__half*>(smem + OFF_MASK);  // [NMASK][128]
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};
  const uint32_t rank = cluster_ctarank();  // 0: the even CTA (issues the MMAs), 1: its pair
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  // the operand this CTA's output channels belong to (c_z = 256: the pair's, constant because the
  // pair count is even; c_z = 128: the CTA's) and the packed weight row of its first signal row
  const int xsel = CZ == 256 ? (pair & 1) : static_cast<int>(rank);
  const int sig_row = CZ == 256 ? 2 * xsel * CC + static_cast<int>(rank) * 128 : 2 * xsel * CC;
  const int ch0 = CZ == 256 ? static_cast<int>(rank) * 128 : 0;  // first output channel of the operand
  const int pih = p.ih >= 2 ? p.ih / 2 : 1;  // this CTA's piece: rows of it (ih >= 2) or one row of 64

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&w_bar, 1);
    mbar_init(&wpair, 2);
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&zfull[s], 1);
      mbar_init(&zempty[s], 1);
      mbar_init(&lnfull[s], 16);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 2 * NEPI);
    }
    for (int k = 0; k < NMASK; ++k) {
      mbar_init(&mfull[k], 8);
      mbar_init(&mempty[k], NEPI);
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
    tmem_alloc_pair(&tmem_base_sh, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  if (warp == 0 && lane == 0) {  // weights are never written by this library: load before the wait
    mbar_arrive_expect_tx(&w_bar, 2 * WBLOCK_BYTES);
    for (int h = 0; h < 2; ++h) {  // h = 0: this CTA's 128 signal rows, 1: its 128 gate rows
      const int row0 = sig_row + h * CC;
      for (int a = 0; a < KATOMS; ++a)
        tma_load_2d(smem + OFF_W + h * WBLOCK_BYTES + a * WATOM_BYTES, &p.tm_w, &w_bar, a * 64, row0);
    }
  }
  griddep_trigger();
  griddep_wait();
  trace_mark_start(p.status, trace_on);
  // Block 0 clears this call's error fields once the previous kernel (which may share the word)
  // has finished; an error another CTA recorded before that survives in the since-reset record.
  if (p.reset_status && blockIdx.x == 0 && threadIdx.x == 0) {
    p.status->code = 0;
    p.status->site = 0;
    p.status->block = 0;
  }

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      if (mbar_wait(&w_bar, 0, ctx, kSiteProducer)) mbar_arrive_cluster(cluster_addr(&wpair, 0));
      uint32_t it = 0;
      for (int tile = pair; tile < p.num_tiles; tile += npairs, ++it) {
        int bb, i0, j0;
        decode_tile<CZ>(p, tile, bb, i0, j0);
        const int pi = i0 + (p.ih >= 2 ? pih * static_cast<int>(rank) : 0);
        const int pj = j0 + (p.ih >= 2 ? 0 : PT * static_cast<int>(rank));
        const uint32_t s = it % NSTAGE, ph = (it / NSTAGE) & 1;
        if (!mbar_wait(&zempty[s], ph ^ 1, ctx, kSiteProducer)) break;
        mbar_arrive_expect_tx(&zfull[s], PIECE_BYTES);
        for (int a = 0; a < KATOMS; ++a)
          tma_load_4d(smem + OFF_A + s * PIECE_BYTES + a * ZATOM_BYTES, &p.tm_z, &zfull[s], a * 64, pj, pi, bb);
      }
      if (abort_sh) {
        mbar_drain(&w_bar, 0, 200000000ull);
        for (uint32_t s = 0; s < NSTAGE; ++s) {
          const uint32_t n_armed = it > s ? (it - s + NSTAGE - 1) / NSTAGE : 0;
          if (n_armed) mbar_drain(&zfull[s], (n_armed - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA): D[slot] = W n^T for both CTAs ----------------
    if (lane == 0 && rank == 0) {
      bool ok = mbar_wait_cl(&wpair, 0, ctx, kSiteMmaW);
      uint32_t it = 0;
      const uint64_t wsd = sdesc_sw128(smem_u32(smem + OFF_W), 16, 1024);
      const uint64_t wgd = sdesc_sw128(smem_u32(smem + OFF_W + WBLOCK_BYTES), 16, 1024);
      for (int tile = pair; ok && tile < p.num_tiles; tile += npairs, ++it) {
        const uint32_t s = it % NSTAGE, ph = (it / NSTAGE) & 1;
        const uint32_t slot = it & 1, sph = (it >> 1) & 1;
        if (!mbar_wait_cl(&lnfull[s], ph, ctx, kSiteMmaLn)) break;
        if (!mbar_wait_cl(&tempty[slot], sph ^ 1, ctx, kSiteMmaSlot)) break;
        tc_fence_after();
        const uint64_t nd = sdesc_sw128(smem_u32(smem + OFF_A + s * PIECE_BYTES), 16, 1024);
        const uint32_t d = tmem_base + slot * 256;
#pragma unroll
        for (int kk = 0; kk < CZ / 16; ++kk) {
          const uint32_t ka = kk >> 2, kb = (kk & 3) * 32;
          umma_f16_pair(d, sdesc_add(wsd, ka * WATOM_BYTES + kb), sdesc_add(nd, ka * ZATOM_BYTES + kb), IDESC,
                        kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < CZ / 16; ++kk) {
          const uint32_t ka = kk >> 2, kb = (kk & 3) * 32;
          umma_f16_pair(d + TILE, sdesc_add(wgd, ka * WATOM_BYTES + kb), sdesc_add(nd, ka * ZATOM_BYTES + kb), IDESC,
                        kk > 0 ? 1u : 0u);
        }
        umma_commit_pair(&zempty[s], 0x3);    // both CTAs' n pieces have been read
        umma_commit_pair(&tfull[slot], 0x3);  // both CTAs' accumulators are complete
      }
      umma_commit_pair(&drain_bar, 0x1);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < EPI_WARP0) {
    // ---------------- LayerNorm of the piece in place + the tile's mask ----------------
    const int t = threadIdx.x - 64;
    const int row = t >> 2, qtr = t & 3;  // lane qtr of the row: its chunks qtr, qtr + 4 of every atom
    uint32_t it = 0, gcount = 0;
    for (int tile = pair; tile < p.num_tiles; tile += npairs, ++it) {
      const uint32_t s = it % NSTAGE, ph = (it / NSTAGE) & 1;
      const uint32_t k = it % NMASK, mph = (it / NMASK) & 1;
      // one thread waits for the piece (and the mask slot), the other LayerNorm warps park on barrier 1
      if (!group_wait(&zfull[s], ph, HAS_MASK ? &mempty[k] : nullptr, mph ^ 1, ctx, kSiteLn, t == 0, 1, 256,
                      gflags + 8, gcount))
        break;
      if (HAS_MASK) {
        if (t < TILE) {  // the tile's 128 positions, in the accumulator's (row-major) order
          int bb, i0, j0;
          decode_tile<CZ>(p, tile, bb, i0, j0);
          const int gi = i0 + (t >> p.log2_jw), gj = j0 + (t & (p.jw - 1));
          __half m = __float2half(0.0f);
          if (gi < p.rows && gj < p.cols) m = p.mask[bb * p.mask_sb + gi * p.mask_si + gj * p.mask_sj];
          maskh[k * TILE + t] = m;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&mfull[k]);
      }
      uint8_t* A = smem + OFF_A + s * PIECE_BYTES;
      // this lane's 8 chunks: atom a, chunk qtr + 4 (h ^ odd) (h = 0, 1) -> u[4 (2a + h) ..].  An odd
      // row starts with the other half of its chunks, so the two rows that share a shared-memory
      // phase (8 lanes) read 8 different 16-byte bank groups.
      const int odd = row & 1;
      uint32_t u[8 * KATOMS];
#pragma unroll
      for (int a = 0; a < KATOMS; ++a)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 v = *reinterpret_cast<const uint4*>(A + a * ZATOM_BYTES + sw128_off(row, qtr + 4 * (h ^ odd)));
          const int e = 4 * (2 * a + h);
          u[e] = v.x;
          u[e + 1] = v.y;
          u[e + 2] = v.z;
          u[e + 3] = v.w;
        }
      // shifted sums around the row's channel 0 (atom 0, chunk 0: lane qtr = 0 holds it in u[0], or
      // in u[4] on an odd row), combined over the row's four lanes by two shuffles
      const uint32_t c0 = odd ? u[4] : u[0];
      const float kshift = __shfl_sync(0xffffffffu, __low2float(*reinterpret_cast<const __half2*>(&c0)), lane & ~3);
      float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int e = 0; e < 8 * KATOMS; ++e) {
        unsigned short lo, hi;
        split_half2(u[e], lo, hi);
        const float2 dd = make_float2(add_f16_f32(lo, -kshift), add_f16_f32(hi, -kshift));
        s1 = __fadd2_rn(s1, dd);
        s2 = __ffma2_rn(dd, dd, s2);
      }
      float t1 = s1.x + s1.y, t2 = s2.x + s2.y;
      t1 += __shfl_xor_sync(0xffffffffu, t1, 1);
      t2 += __shfl_xor_sync(0xffffffffu, t2, 1);
      t1 += __shfl_xor_sync(0xffffffffu, t1, 2);
      t2 += __shfl_xor_sync(0xffffffffu, t2, 2);
      const float m1 = t1 * (1.0f / CZ);
      const float var = fmaxf(t2 * (1.0f / CZ) - m1 * m1, 0.0f);
      const float mean = kshift + m1;
      const float rs = rsqrtf(var + 1e-5f);
      const float2 r2 = make_float2(rs, rs);
      const LnParSmemHalf lpar{par, par + CZ};
#pragma unroll
      for (int a = 0; a < KATOMS; ++a)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c16 = qtr + 4 * (h ^ odd);  // chunk within the atom: channels 64 a + 8 c16 ..
          float g[8], b[8];
          lpar(8 * a + c16, g, b);
          const int e0 = 4 * (2 * a + h);
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            unsigned short lo, hi;
            split_half2(u[e0 + e], lo, hi);
            const float2 dd = __fmul2_rn(make_float2(add_f16_f32(lo, -mean), add_f16_f32(hi, -mean)), r2);
            const float2 y = __ffma2_rn(dd, make_float2(g[2 * e], g[2 * e + 1]), make_float2(b[2 * e], b[2 * e + 1]));
            o[e] = pack_half2(y.x, y.y);
          }
          *reinterpret_cast<uint4*>(A + a * ZATOM_BYTES + sw128_off(row, c16)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      fence_proxy_async_smem();  // generic-proxy writes to this CTA's shared memory -> the paired MMA's reads
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_smem(cluster_addr(&lnfull[s], 0));
    }
  } else {
    // ---------------- epilogue: gate, mask, channel-major store ----------------
    const int grp = (warp - EPI_WARP0) >> 2;  // positions [32 grp, 32 grp + 32) of the tile
    const int q = warp & 3;                   // TMEM lane quadrant = channels [32q, 32q+32) of the CTA's half
    const int chl = q * 32 + lane;
    const int ch = ch0 + chl;  // channel of the operand
    uint8_t* stg = smem + OFF_STG + (warp - EPI_WARP0) * WSTG_BYTES;
    // byte offsets in the staging block of this thread's two 16-byte chunks c of compute step
    // st (positions 16 st + 8 c ..), matching the store box and its swizzle (as in K1)
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
    if (HAS_BIAS) {  // packed order: this CTA's signal rows start at sig_row, its gate rows c later
      bs = __ldg(p.bias + sig_row + chl);
      bgt = __ldg(p.bias + sig_row + CC + chl);
    }
    const float2 bs2 = make_float2(bs, bs), bg2 = make_float2(bgt, bgt);
    const CUtensorMap* tm = xsel == 0 ? &p.tm_a : &p.tm_b;
    uint32_t it = 0, gcount = 0;
    const bool leader = ((warp - EPI_WARP0) & 3) == 0 && lane == 0;
    for (int tile = pair; tile < p.num_tiles; tile += npairs, ++it) {
      int bb, i0, j0;
      decode_tile<CZ>(p, tile, bb, i0, j0);
      const uint32_t slot = it & 1, sph = (it >> 1) & 1;
      const uint32_t k = it % NMASK, mph = (it / NMASK) & 1;
      // one thread of the group waits, the other warps park on barrier 2 + grp
      if (!group_wait_cl(&tfull[slot], sph, HAS_MASK ? &mfull[k] : nullptr, mph, ctx, kSiteEpilogue, leader, 2 + grp,
                         128, gflags + 2 * grp, gcount))
        break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + slot * 256 + 32 * grp;
      const __half* mrow = maskh + k * TILE + 32 * grp;
#pragma unroll 1
      for (int pb = 0; pb < SPOS; pb += POS) {
        uint32_t sg[16], gt[16];
        tmem_ld16(taddr + pb, sg);
        tmem_ld16(taddr + TILE + pb, gt);
        tmem_wait_ld16x2(sg, gt);
        if (pb == SPOS - POS) {  // this group's columns of the slot have been read
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster_smem(cluster_addr(&tempty[slot], 0));
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
            const int tp = 32 * grp;  // tile position of the first of these 32
            tma_store_3d(tm, stg, j0 + (tp & (p.jw - 1)), i0 + (tp >> p.log2_jw), bb * CC + ch - lane);
            bulk_commit();
          }
        }
      }
      if (HAS_MASK) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&mempty[k]);
      }
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  trace_mark_end(p.status, trace_on);
  // Neither CTA leaves (or frees the pair's TMEM) while the other can still arrive on its
  // barriers or run a paired MMA over its shared memory.
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace k1p
}  // namespace tmu
