// K3P: K3 for c_z = c = 256 (mlx_trunk.py:4) on CTA pairs.  Same arithmetic as K3 (mlx_trunk.py:
// 89-90,94-95; mlx_trunk_kernels.py:107-147,165-190,221-227):
//   m = fp16(LN_mix(x^T)), mixed = fp16(m @ w_emit [+ b]), g = fp16(n @ w_out_gate [+ b]),
//   z' = fp16(z + mixed * sigmoid(g)),  n = fp16(LN(z; norm_start)).
//
// w_emit and w_out_gate are 2 x 256 x 256 fp16 = 256 KB, more than one SM's shared memory.  A
// cluster of two CTAs on two SMs shares each tile instead, through MMAs that span both SMs
// (tcgen05 .cta_group::2, M = 256 output channels): CTA r keeps rows [128 r, 128 r + 128) of
// both matrices resident in its tensor memory (the A operand's half, which the MMA reads from
// TMEM, so the MMAs take only the activations from shared memory), normalises ITS 32 of the
// tile's 64 positions (the B operand's half), and receives in its TMEM the accumulators of its
// 128 output channels
// for all 64 positions.  So every LayerNorm is computed once (a design that splits the output
// channels over two independent CTAs computes each twice), and one MMA instruction covers
// 256 x 64 outputs.
//
// Tile = 64 positions of the pair grid as a 2 x 32 block (CTA r: row i0 + r) or a 1 x 64 block
// (CTA r: columns j0 + 32 r ..), so each CTA's piece is one row of 32 positions.  Per CTA and
// tile (14 warps, 448 threads):
//   warp 0      TMA: per tile its piece of x (channel-major [256][32], 64B-swizzled, 16 KB) and
//               of z ([4 atoms][32 positions][128 B], 16 KB), 4 stages, and the residual block
//               z[64 positions][its 128 channels] (16 KB), 4 stages
//   warp 1      TMEM (512 columns for the pair: 2 accumulator slots x 128, then w_emit's and
//               w_gate's rows) and, in the even CTA, the MMA thread: emit and gate chains,
//               M = 256, N = 64, K = 256, A from TMEM
//   warps 2-5   A1 = fp16(LN_mix(x column)) in place over the x piece (ldmatrix.trans
//               transpose, four 64-channel atoms combined by the parallel-variance formula)
//   warps 6-9   A2 = fp16(LN_in(z row)) in place over the z piece
//   warps 10-13 first the weights into TMEM (a thread per output-channel row, from global
//               memory, before the dependency wait); then the epilogue, TMEM lane quadrant warp
//               mod 4: z' = z + m * sigmoid(g) over the residual block in shared memory, then
//               one TMA store of the block.
// Cross-CTA traffic is mbarrier signals only: the LayerNorm warps of both CTAs arrive on the
// even CTA's operand barrier, the epilogue warps of both on its accumulator-free barrier, and the
// MMA thread's commits arrive in both CTAs (multicast).  A2 in place frees a buffer that the
// residual block reuses: the residual is reloaded from z (an L2 hit) for all 64 positions of
// this CTA's channels.  z_out must not alias z (the pair's other CTA still reads z's channels
// that this CTA writes).
//
// With the weights in shared memory (an earlier form), every M = 256, N = 64 MMA re-read 4 KB
// of weights per CTA against 1 KB of activations: shared-memory bandwidth kept the paired MMAs
// well below the tensor rate, and the 128 KB left room for only two operand and residual stages.
#pragma once

#include "tmu_common.cuh"

namespace tmu {
namespace k3p {

constexpr int CZ = 256;
constexpr int CC = 256;
constexpr int TILE = 64;                        // positions per pair tile
constexpr int PT = 32;                          // positions per CTA
constexpr int ATOM_BYTES = PT * 128;            // activation atoms: 32 rows x 128 B
constexpr int PIECE_BYTES = PT * 256 * 2;       // 32 positions x 256 channels
constexpr int RATOM_BYTES = TILE * 128;         // residual atoms: 64 rows x 128 B
constexpr int RES_BYTES = 2 * RATOM_BYTES;      // 64 positions x 128 channels
constexpr int NS = 4;                           // operand stages (x and z pieces)
constexpr int NR = 4;                           // residual stages
constexpr int OFF_X = 0;                           // NS stages: the x piece, then A1 in place
constexpr int OFF_Z = OFF_X + NS * PIECE_BYTES;    // NS stages: the z piece, then A2 in place
constexpr int OFF_R = OFF_Z + NS * PIECE_BYTES;    // NR stages: residual z, then z' in place
constexpr int OFF_RED = OFF_R + NR * RES_BYTES;    // float2 [4 parts][32 positions]: LN_mix partials
constexpr int OFF_REDI = OFF_RED + 4 * PT * 8;     // the same for LN_in
constexpr int OFF_BAR = OFF_REDI + 4 * PT * 8;
constexpr int SMEM_BYTES = OFF_BAR + 512;
constexpr int kThreads = 448;
// TMEM: columns [0, 256) two accumulator slots (emit and gate, 64 positions each), [256, 384)
// this CTA's 128 rows of w_emit and [384, 512) of w_gate as the MMA's A operand (K = 256 at two
// fp16 per column)
constexpr int TMEM_COLS = 512;
constexpr int TM_WE = 256, TM_WG = 384;
static_assert(SMEM_BYTES <= 232448, "K3P shared memory exceeds the per-block limit");

struct Params {
  CUtensorMap tm_z;   // z [B, rows, cols, 256]: box {64, 32, 1, 1}, 128B swizzle (a CTA's piece, per atom)
  CUtensorMap tm_r;   // z, box {64, jw, ih, 1} (the tile's 64 positions, per atom)
  CUtensorMap tm_zo;  // z_out, box {64, jw, ih, 1} (store)
  CUtensorMap tm_x;   // x [B*256, rows, pitch]: box {32, 1, 256}, 64B swizzle
  const __half* w_emit;  // [256 out][256 in] (nn.Linear): row r = output channel r
  const __half* w_gate;
  const __half* ln_in_w;
  const __half* ln_in_b;
  const __half* ln_mix_w;
  const __half* ln_mix_b;
  const float* b_emit;  // [256] or null
  const float* b_gate;  // [256] or null
  float mix_eps;
  int rows, cols, ih, jw, tiles_i, tiles_j, num_tiles;  // tile = ih x jw = 2 x 32 or 1 x 64
  DeviceStatus* status;
  unsigned long long timeout_ns;
};

enum Site : unsigned int {
  kSiteProd = 0x321, kSiteProdR = 0x322, kSiteMix = 0x323, kSiteIn = 0x324, kSiteMmaW = 0x325,
  kSiteMmaA = 0x326, kSiteMmaT = 0x327, kSiteEpilogue = 0x328
};

__device__ __forceinline__ void decode_tile(const Params& p, int tile, int& bb, int& i0, int& j0) {
  const int per_b = p.tiles_i * p.tiles_j;
  bb = tile / per_b;
  const int r = tile - bb * per_b;
  i0 = (r / p.tiles_j) * p.ih;
  j0 = (r % p.tiles_j) * p.jw;
}

template <bool HAS_BIAS>
__global__ void __launch_bounds__(kThreads, 1) emit_residual_pair_kernel(const __grid_constant__ Params p) {
  const bool trace_on = trace_enabled(p.status);
  constexpr uint32_t IDESC = idesc_f16_f32(256, TILE, false, false);
  extern __shared__ uint8_t smem[];
  // Both CTAs of a cluster take the same branch here (the alignment of the dynamic buffer is a
  // property of the kernel), so neither can be left waiting at the cluster barriers below.
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(p.status, kStatusLayout, 0x32f);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t& wpair = bars[1];     // even CTA: both CTAs' weight rows are in TMEM (8 arrivals)
  uint64_t* xfull = bars + 2;    // [NS]
  uint64_t* zfull = bars + 6;    // [NS]
  uint64_t* rfull = bars + 10;   // [NR]
  uint64_t* rempty = bars + 14;  // [NR] the epilogue's store has read the residual stage
  uint64_t* afull = bars + 18;   // [NS] even CTA: A1 and A2 of both CTAs (16 arrivals)
  uint64_t* aempty = bars + 22;  // [NS] the paired MMAs have read A1 and A2 (multicast commit)
  uint64_t* tfull = bars + 26;   // [2] the accumulator slot is complete (multicast commit)
  uint64_t* tempty = bars + 28;  // [2] even CTA: both CTAs' epilogues have read the slot (8 arrivals)
  uint64_t& drain_bar = bars[30];
  uint32_t& tmem_base_sh = *reinterpret_cast<uint32_t*>(bars + 31);
  volatile int& abort_sh = *reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(bars + 31) + 4);
  volatile int* ok_sh = reinterpret_cast<volatile int*>(bars + 32);  // [3][2]
  float2* rd = reinterpret_cast<float2*>(smem + OFF_RED);
  float2* rdi = reinterpret_cast<float2*>(smem + OFF_REDI);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx ctx{p.status, &abort_sh, p.timeout_ns};
  const uint32_t rank = cluster_ctarank();  // 0: the even CTA (issues the MMAs), 1: its pair
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&wpair, 8);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&zfull[s], 1);
      mbar_init(&afull[s], 16);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < NR; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 8);
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_z);
    tma_prefetch_desc(&p.tm_r);
    tma_prefetch_desc(&p.tm_zo);
    tma_prefetch_desc(&p.tm_x);
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
  if (warp >= 10) {
    // The weights (never written by this library: loaded before the dependency wait) go to TMEM
    // as the MMA's A operand: each epilogue warp writes its lane quadrant, thread = one output
    // channel row, 512 B of w_emit and of w_gate straight from global memory.  Resident for the
    // kernel, so the MMAs read only the activations from shared memory.
    const int q = warp & 3;
    const size_t row = static_cast<size_t>(rank) * 128 + q * 32 + lane;
    const uint32_t tq = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
    for (int m = 0; m < 2; ++m) {
      const uint4* src = reinterpret_cast<const uint4*>((m == 0 ? p.w_emit : p.w_gate) + row * CZ);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {  // 32 columns (64 K elements) at a time
        uint32_t r[32];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint4 v = __ldg(src + 8 * c + e);
          r[4 * e] = v.x, r[4 * e + 1] = v.y, r[4 * e + 2] = v.z, r[4 * e + 3] = v.w;
        }
        tmem_st32(tq + (m == 0 ? TM_WE : TM_WG) + 32 * c, r);
      }
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(cluster_addr(&wpair, 0));  // once per kernel
  }
  griddep_trigger();
  griddep_wait();
  trace_mark_start(p.status, trace_on);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0, nxz = 0, nr = 0;
      for (int tile = pair; tile < p.num_tiles; tile += npairs, ++it) {
        int bb, i0, j0;
        decode_tile(p, tile, bb, i0, j0);
        const int pi = i0 + (p.ih == 2 ? static_cast<int>(rank) : 0);
        const int pj = j0 + (p.ih == 2 ? 0 : PT * static_cast<int>(rank));
        const uint32_t s = it % NS, ph = (it / NS) & 1;
        const uint32_t rs = it % NR, rph = (it / NR) & 1;
        // the paired MMAs of this stage's previous tile have read A1 and A2 (both in place)
        if (!mbar_wait(&aempty[s], ph ^ 1, ctx, kSiteProd)) break;
        mbar_arrive_expect_tx(&xfull[s], PIECE_BYTES);
        tma_load_3d(smem + OFF_X + s * PIECE_BYTES, &p.tm_x, &xfull[s], pj, pi, bb * CC);
        mbar_arrive_expect_tx(&zfull[s], PIECE_BYTES);
        for (int a = 0; a < 4; ++a)
          tma_load_4d(smem + OFF_Z + s * PIECE_BYTES + a * ATOM_BYTES, &p.tm_z, &zfull[s], a * 64, pj, pi, bb);
        ++nxz;
        if (!mbar_wait(&rempty[rs], rph ^ 1, ctx, kSiteProdR)) break;
        mbar_arrive_expect_tx(&rfull[rs], RES_BYTES);
        for (int k = 0; k < 2; ++k)
          tma_load_4d(smem + OFF_R + rs * RES_BYTES + k * RATOM_BYTES, &p.tm_r, &rfull[rs], (2 * rank + k) * 64, j0,
                      i0, bb);
        ++nr;
      }
      if (abort_sh) {
        for (uint32_t s = 0; s < NS; ++s) {
          const uint32_t na = nxz > s ? (nxz - s + NS - 1) / NS : 0;
          if (na) {
            mbar_drain(&xfull[s], (na - 1) & 1, 200000000ull);
            mbar_drain(&zfull[s], (na - 1) & 1, 200000000ull);
          }
        }
        for (uint32_t s = 0; s < NR; ++s) {
          const uint32_t nra = nr > s ? (nr - s + NR - 1) / NR : 0;
          if (nra) mbar_drain(&rfull[s], (nra - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA): emit and gate chains for both CTAs ----------------
    if (lane == 0 && rank == 0) {
      bool ok = mbar_wait_cl(&wpair, 0, ctx, kSiteMmaW);  // both CTAs' weight rows are in TMEM
      tc_fence_after();
      uint32_t it = 0;
      for (int tile = pair; ok && tile < p.num_tiles; tile += npairs, ++it) {
        const uint32_t s = it % NS, ph = (it / NS) & 1;  // operand stage
        const uint32_t a = it & 1, aph = (it >> 1) & 1;  // accumulator slot
        if (!mbar_wait_cl(&afull[s], ph, ctx, kSiteMmaA)) break;
        if (!mbar_wait_cl(&tempty[a], aph ^ 1, ctx, kSiteMmaT)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * 128;
        const uint64_t a1d = sdesc_sw128(smem_u32(smem + OFF_X + s * PIECE_BYTES), 16, 1024);
        const uint64_t a2d = sdesc_sw128(smem_u32(smem + OFF_Z + s * PIECE_BYTES), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {  // K step kk: 8 TMEM columns of the weights
          const uint32_t ka = kk >> 2, kb = (kk & 3) * 32;
          umma_f16_pair_ts(d, tmem_base + TM_WE + 8 * kk, sdesc_add(a1d, ka * ATOM_BYTES + kb), IDESC,
                           kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          const uint32_t ka = kk >> 2, kb = (kk & 3) * 32;
          umma_f16_pair_ts(d + TILE, tmem_base + TM_WG + 8 * kk, sdesc_add(a2d, ka * ATOM_BYTES + kb), IDESC,
                           kk > 0 ? 1u : 0u);
        }
        umma_commit_pair(&aempty[s], 0x3);  // A1 and A2 of both CTAs have been read
        umma_commit_pair(&tfull[a], 0x3);   // both CTAs' accumulators are complete
      }
      umma_commit_pair(&drain_bar, 0x1);
      mbar_drain(&drain_bar, 0, 200000000ull);
    }
  } else if (warp < 10) {
    // ---------------- LayerNorms: warps 2-5 LN_mix (x -> A1), warps 6-9 LN_in (z -> A2) ----------------
    const bool mix = warp < 6;
    const int grp = mix ? 0 : 1;
    const int t = threadIdx.x - (mix ? 64 : 192);
    const int row = t & 31, part = t >> 5;  // part = this warp's 64-channel atom
    const uint32_t bar_id = 1 + grp;
    const LnParHalf par{p.ln_in_w, p.ln_in_b};
    // LN_mix parameters of this lane: channel pairs 64 part + 32g + 8j + 2(t%4) (g < 2, j < 4)
    uint32_t gmw[8], bmw[8];
    if (mix) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = 64 * part + 32 * (e >> 2) + 8 * (e & 3) + 2 * (lane & 3);
        gmw[e] = __ldg(reinterpret_cast<const unsigned int*>(p.ln_mix_w + c));
        bmw[e] = __ldg(reinterpret_cast<const unsigned int*>(p.ln_mix_b + c));
      }
    }
    uint32_t it = 0;
    for (int tile = pair; tile < p.num_tiles; tile += npairs, ++it) {
      const uint32_t s = it % NS, ph = (it / NS) & 1;
      // one thread waits (bounded) and shares the verdict, so the group meets at every barrier
      if (t == 0) {
        const bool ok = mbar_wait(mix ? &xfull[s] : &zfull[s], ph, ctx, mix ? kSiteMix : kSiteIn);
        ok_sh[2 * grp + (it & 1)] = ok ? 1 : 0;
      }
      named_bar_sync(bar_id, 128);
      if (!ok_sh[2 * grp + (it & 1)]) break;
      if (mix) {
        // The x piece: [channel][32 positions], 64 B per channel, the 16-byte chunk m (positions
        // 8m..8m+7) of channel ch at chunk m ^ ((ch >> 1) & 3).  ldmatrix.trans of the 8 x 8 block
        // (channels 8cb.., positions 8m..) gives lane t channels 8cb + 2(t%4), +1 of position
        // 8m + t/4 (lane t addresses channel 32g + t of this warp's atom; eight channel rows fall
        // in eight bank groups).
        const uint32_t xs = smem_u32(smem + OFF_X + s * PIECE_BYTES);
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
            const float2 dd = make_float2(add_f16_f32(lo, -k), add_f16_f32(hi, -k));
            s1 = __fadd2_rn(s1, dd);
            s2 = __ffma2_rn(dd, dd, s2);
          }
          float t1 = s1.x + s1.y, t2 = s2.x + s2.y;
          t1 += __shfl_xor_sync(0xffffffffu, t1, 1);
          t2 += __shfl_xor_sync(0xffffffffu, t2, 1);
          t1 += __shfl_xor_sync(0xffffffffu, t1, 2);
          t2 += __shfl_xor_sync(0xffffffffu, t2, 2);
          if ((lane & 3) == 0) rd[part * PT + 8 * m + (lane >> 2)] = make_float2(k + t1 * (1.0f / 64), t2 - t1 * t1 * (1.0f / 64));
        }
        named_bar_sync(bar_id, 128);  // every atom's partials are written; every x value is in registers
        uint8_t* A1 = smem + OFF_X + s * PIECE_BYTES;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          // the four atoms combined (Chan et al.): mean of the means, M2 = sum M2_a + 64 sum (mean_a - mean)^2
          const int pos = 8 * m + (lane >> 2);
          const float2 a0 = rd[pos], a1 = rd[PT + pos], a2 = rd[2 * PT + pos], a3 = rd[3 * PT + pos];
          const float mean = 0.25f * ((a0.x + a1.x) + (a2.x + a3.x));
          const float d0 = a0.x - mean, d1 = a1.x - mean, d2 = a2.x - mean, d3 = a3.x - mean;
          const float m2 = (a0.y + a1.y) + (a2.y + a3.y) + 64.0f * ((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3));
          const float rs = rsqrtf(fmaxf(m2 * (1.0f / 256), 0.0f) + p.mix_eps);
          const float2 r2 = make_float2(rs, rs);
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              unsigned short lo, hi;
              split_half2(u[m][4 * g + j], lo, hi);
              const float2 dd = __fmul2_rn(make_float2(add_f16_f32(lo, -mean), add_f16_f32(hi, -mean)), r2);
              const float2 gv = unpack_half2(gmw[4 * g + j]), bv = unpack_half2(bmw[4 * g + j]);
              const float2 y = __ffma2_rn(dd, gv, bv);
              o[j] = pack_half2(y.x, y.y);
            }
            // A1 atom `part` (32 rows x 128 B, K-major 128B-swizzled): lane l gives the row of
            // position 8m + l%8 in chunk 4g + l/8
            const uint32_t row8 = lane & 7;
            stsm_x4(smem_u32(A1) + part * ATOM_BYTES + (8 * m + row8) * 128 + 16 * ((4 * g + (lane >> 3)) ^ row8), o[0],
                    o[1], o[2], o[3]);
          }
        }
      } else {
        // LN_in of this CTA's 32 positions in place over the z piece (A2): a warp per 64-channel
        // atom, the four partial sums of a row meeting in shared memory
        uint8_t* Zp = smem + OFF_Z + s * PIECE_BYTES;
        const float shift = ln_row_shift(Zp, row);
        rdi[part * PT + row] = ln_atom_sums(Zp, ATOM_BYTES, row, part, shift);
        named_bar_sync(bar_id, 128);
        const float2 s0 = rdi[row], s1 = rdi[PT + row], s2 = rdi[2 * PT + row], s3 = rdi[3 * PT + row];
        const float2 mr = ln256_moments(make_float2(s0.x + s1.x, s0.y + s1.y), make_float2(s2.x + s3.x, s2.y + s3.y),
                                        shift, 1e-5f);
        ln_atom_apply(Zp, Zp, ATOM_BYTES, row, part, mr.x, mr.y, par);
      }
      fence_proxy_async_smem();  // generic-proxy writes to this CTA's shared memory -> the paired MMA's reads
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_smem(cluster_addr(&afull[s], 0));
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;                    // TMEM lane quadrant this warp may access
    const int chl = q * 32 + lane;             // this thread's output channel within the CTA's half
    const int ch = static_cast<int>(rank) * 128 + chl;
    const uint32_t zoff = (chl >> 6) * RATOM_BYTES + (chl & 7) * 2;  // + sw128_off(position, chunk)
    const uint32_t chunk = (chl & 63) >> 3;
    float be = 0.f, bgv = 0.f;
    if (HAS_BIAS) {
      be = __ldg(p.b_emit + ch);
      bgv = __ldg(p.b_gate + ch);
    }
    const float2 be2 = make_float2(be, be), bg2 = make_float2(bgv, bgv);
    uint32_t it = 0;
    for (int tile = pair; tile < p.num_tiles; tile += npairs, ++it) {
      int bb, i0, j0;
      decode_tile(p, tile, bb, i0, j0);
      const uint32_t a = it & 1, aph = (it >> 1) & 1;    // accumulator slot
      const uint32_t rs = it % NR, rph = (it / NR) & 1;  // residual stage
      if (warp == 10 && lane == 0) {
        bool ok = mbar_wait_cl(&tfull[a], aph, ctx, kSiteEpilogue);
        ok = ok && mbar_wait(&rfull[rs], rph, ctx, kSiteEpilogue);
        ok_sh[4 + (it & 1)] = ok ? 1 : 0;
      }
      named_bar_sync(3, 128);
      if (!ok_sh[4 + (it & 1)]) break;
      tc_fence_after();
      uint8_t* Rs = smem + OFF_R + rs * RES_BYTES;
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + a * 128;
#pragma unroll 1
      for (int pb = 0; pb < TILE; pb += 16) {
        uint32_t em[16], gt[16];
        tmem_ld16(trow + pb, em);
        tmem_ld16(trow + TILE + pb, gt);
        tmem_wait_ld16x2(em, gt);
        if (pb == TILE - 16) {  // the slot has been read: hand it back to the MMA thread
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster_smem(cluster_addr(&tempty[a], 0));
        }
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          __half* z0 = reinterpret_cast<__half*>(Rs + zoff + sw128_off(pb + i, chunk));
          __half* z1 = reinterpret_cast<__half*>(Rs + zoff + sw128_off(pb + i + 1, chunk));
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
        for (int k = 0; k < 2; ++k)
          tma_store_4d(&p.tm_zo, Rs + k * RATOM_BYTES, (2 * rank + k) * 64, j0, i0, bb);
        bulk_commit();
        // release the PREVIOUS tile's residual stage once its store has read it (long done): the
        // group does not wait for this tile's store to read its block (0.45 us a tile when it did)
        if (it > 0) {
          bulk_wait_read<1>();
          mbar_arrive(&rempty[(it - 1) % NR]);
        }
      }
    }
    if (warp == 10 && lane == 0) bulk_wait<0>();
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

}  // namespace k3p
}  // namespace tmu
