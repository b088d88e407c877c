// Host side of the C ABI declared in include/tmu.h: argument checks, TMA tensor maps, tile
// shapes, launches and the device status word.  Nothing here allocates device memory or
// synchronises a stream (except tmu_read_status, whose job is to).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <string>

#include "k1_project.cuh"
#include "k1p_project.cuh"
#include "k3p_emit.cuh"
#include "k2_contract.cuh"
#include "k3_emit.cuh"
#include "k4_transition.cuh"
#include "k5_disto.cuh"
#include "k6_gemm.cuh"
#include "tmu.h"

using namespace tmu;

namespace {

thread_local std::string g_last_error;
unsigned long long g_timeout_ns = 2000000000ull;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

constexpr int kMaxDevices = 64;
int g_num_sms[kMaxDevices] = {0};
unsigned long long g_attr_done[kMaxDevices] = {0};

int fail(int code, const char* what) {
  g_last_error = what;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return TMU_ERR_CUDA;
}

int get_encoder() {
  static std::once_flag once;
  static int st = TMU_OK;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
      st = TMU_ERR_DRIVER;
      g_last_error = "cuTensorMapEncodeTiled entry point not available";
    } else {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  return st;
}

// Start address of the allocation that contains `ptr` (cuMemGetAddressRange through the runtime's
// driver entry point, as for the tensor-map encoder: the library does not link libcuda).
int allocation_base(const void* ptr, CUdeviceptr* base) {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 3020, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  });
  if (fn == nullptr) return fail(TMU_ERR_DRIVER, "cuMemGetAddressRange entry point not available");
  size_t size = 0;
  if (fn(base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(TMU_ERR_INVALID_ARGUMENT, "pointer is not inside a device allocation");
  return TMU_OK;
}

int encode_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
               const uint32_t* box, CUtensorMapSwizzle sw) {
  int st = get_encoder();
  if (st != TMU_OK) return st;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides[i];
  }
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
                        d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d), rank %d", static_cast<int>(r), rank);
    return fail(TMU_ERR_DRIVER, buf);
  }
  return TMU_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int row_pitch(int L) { return (L + 7) & ~7; }

// A tile of `tile` (128 or 64) positions as an ih x jw block of a rows x cols pair grid, jw >= 8,
// minimising padding.
void choose_tile(int rows, int cols, int& ih, int& jw, int tile = 128) {
  static const int widths[5] = {128, 64, 32, 16, 8};
  long long best = -1;
  for (int wi : widths) {
    if (wi > tile || tile / wi > 16) continue;  // 128: 1x128 .. 16x8; 64: 1x64 .. 8x8
    const int hi = tile / wi;
    const long long area = static_cast<long long>((rows + hi - 1) / hi) * hi * ((cols + wi - 1) / wi) * wi;
    if (best < 0 || area < best) {
      best = area;
      ih = hi;
      jw = wi;
    }
  }
}

// K1's tile: measured per position, K1 is fastest on 1 x 128 tiles (3.1-3.7 TB/s at L = 1024-
// 2048) and slower the narrower the tile (L = 1032: 8 x 16 tiles 1.39x the 1 x 128 cost per
// position, 4 x 32 1.1x; L = 1544 and 2056: 8 x 16 and 4 x 32 tiles 1.4-1.8x), the channel-major
// stores covering fewer positions per row.  Each shape is charged its relative cost per
// position, so some padding buys the wide tiles.  Below 512 x 512 positions the outputs stay in
// L2 and the least padding measured best (L = 238: 8 x 16 tiles 2 % faster than 1 x 128).
void choose_tile_k1(int rows, int cols, int& ih, int& jw) {
  static const int widths[5] = {128, 64, 32, 16, 8};
  static const int weight[5] = {20, 22, 25, 28, 32};  // relative cost per position, x 20
  const bool dram = static_cast<long long>(rows) * cols >= 512ll * 512;
  long long best = -1;
  for (int w = 0; w < 5; ++w) {
    const int wi = widths[w], hi = 128 / wi;
    const long long area = static_cast<long long>((rows + hi - 1) / hi) * hi * ((cols + wi - 1) / wi) * wi;
    const long long cost = area * (dram ? weight[w] : 1);
    if (best < 0 || cost < best) {
      best = cost;
      ih = hi;
      jw = wi;
    }
  }
}

// K3's tile: as choose_tile, but a shape with jw >= 32 (whose x tile is transposed by ldmatrix)
// is charged 10 % less per position than the narrower shapes (2-byte gather), the measured
// difference in K3's time per tile, so a little padding buys the faster path.
void choose_tile_k3(int rows, int cols, int& ih, int& jw) {
  static const int widths[5] = {128, 64, 32, 16, 8};
  long long best = -1;
  for (int wi : widths) {
    const int hi = 128 / wi;
    const long long area = static_cast<long long>((rows + hi - 1) / hi) * hi * ((cols + wi - 1) / wi) * wi;
    const long long cost = area * (wi >= 32 ? 10 : 11);
    if (best < 0 || cost < best) {
      best = cost;
      ih = hi;
      jw = wi;
    }
  }
}

struct Dev {
  int id;
  int sms;
};

int current_device(Dev& d, unsigned long long attr_bit, const void* kernel, int smem) {
  cudaError_t e = cudaGetDevice(&d.id);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (d.id < 0 || d.id >= kMaxDevices) return fail(TMU_ERR_INVALID_ARGUMENT, "device id out of range");
  if (g_num_sms[d.id] == 0) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d.id);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    g_num_sms[d.id] = n;
  }
  d.sms = g_num_sms[d.id];
  if (attr_bit != 0 && !(g_attr_done[d.id] & attr_bit)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    g_attr_done[d.id] |= attr_bit;
  }
  return TMU_OK;
}

int check_sizes(int B, int L, int c_z, int c) {
  if (B < 1 || L < 1) return fail(TMU_ERR_INVALID_ARGUMENT, "B and L must be positive");
  if (c_z != c || (c != 128 && c != 256)) return fail(TMU_ERR_UNSUPPORTED, "c_z == c, 128 or 256, is built");
  if (L > 8192) return fail(TMU_ERR_UNSUPPORTED, "L > 8192");
  if (static_cast<long long>(B) * c > 65535) return fail(TMU_ERR_UNSUPPORTED, "B*c > 65535");
  return TMU_OK;
}

// The c_z = 256 emit kernel splits each tile's output channels over two CTAs, so one CTA may write
// z' while the other still reads z: an in-place (or overlapping) update is rejected up front.
int check_wide_alias(const void* z, const void* z_out, int B, int L, int c_z) {
  if (c_z != 256) return TMU_OK;
  const uintptr_t bytes = static_cast<uintptr_t>(B) * L * L * 256 * 2;
  const uintptr_t zi = reinterpret_cast<uintptr_t>(z), zo = reinterpret_cast<uintptr_t>(z_out);
  if (zi < zo + bytes && zo < zi + bytes)
    return fail(TMU_ERR_INVALID_ARGUMENT, "c_z = 256: z_out must not overlap z (no in-place update)");
  return TMU_OK;
}

int check_weights(const tmu_trimul_weights* w, bool k1, bool k3) {
  if (w == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "weights is NULL");
  if (k1 && (!w->ln_in_w || !w->ln_in_b || !w->w_proj)) return fail(TMU_ERR_INVALID_ARGUMENT, "K1 weights missing");
  if (k3 && (!w->ln_in_w || !w->ln_in_b || !w->ln_mix_w || !w->ln_mix_b || !w->w_emit || !w->w_gate))
    return fail(TMU_ERR_INVALID_ARGUMENT, "K3 weights missing");
  const void* al[] = {w->ln_in_w, w->ln_in_b, w->w_proj, w->ln_mix_w, w->ln_mix_b, w->w_emit, w->w_gate};
  for (const void* p : al)
    if (p != nullptr && !aligned16(p)) return fail(TMU_ERR_MISALIGNED, "weight pointer not 16-byte aligned");
  return TMU_OK;
}

// Launch with programmatic stream serialisation: the kernel may begin (prologue: barriers,
// TMEM, weight loads) while the previous kernel in the stream drains; each kernel waits with
// griddepcontrol.wait before touching data another kernel produces or consumes.
template <typename P>
cudaError_t launch_pdl(void (*kern)(P), int grid, int block, int smem, cudaStream_t stream, const P& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// A launch of clusters of two CTAs (CTA pairs), chained like launch_pdl.
template <typename P>
cudaError_t launch_pdl_pair(void (*kern)(P), int grid, int block, int smem, cudaStream_t stream, const P& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// How many CTA pairs of `kern` can be resident at once on the current device (cached per device
// and kernel by the caller): pairs need two SMs of one GPC, so this can be below SMs / 2.
template <typename P>
int max_resident_pairs(void (*kern)(P), int block, int smem) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();  // clear the error: fall back to one pair per two SMs
    return 0;
  }
  return n;
}

// A pair tensor [B, rows, cols, cz] with contiguous channels and arbitrary element strides
// (z, or a transposed view of a received slab), plus the element strides of its mask.
struct PairGeom {
  int B, rows, cols;
  long long sb, sr, sc;
  long long msb, msr, msc;
  int cz;
};

PairGeom square_geom(int B, int L, int cz) {
  return PairGeom{B, L, L, 1LL * cz * L * L, 1LL * cz * L, cz, 1LL * L * L, L, 1, cz};
}

template <int CZ>
int launch_k1p(const void* z, const void* mask, const tmu_trimul_weights* w, const PairGeom& g, void* a, void* b,
               DeviceStatus* status, cudaStream_t stream, bool reset_status);

int launch_k1(const void* z, const void* mask, const tmu_trimul_weights* w, const PairGeom& g, void* a, void* b,
              DeviceStatus* status, cudaStream_t stream, bool reset_status = false) {
  if (g.cz == 256) return launch_k1p<256>(z, mask, w, g, a, b, status, stream, reset_status);
  const bool hb = w->b_proj != nullptr, hm = mask != nullptr;
  void (*kern)(k1::Params) = hb ? (hm ? k1::project_gate_kernel<true, true> : k1::project_gate_kernel<true, false>)
                                : (hm ? k1::project_gate_kernel<false, true> : k1::project_gate_kernel<false, false>);
  Dev dev;
  int st = current_device(dev, 1u << (8 + (hb ? 2 : 0) + (hm ? 1 : 0)), reinterpret_cast<const void*>(kern),
                          k1::SMEM_BYTES);
  if (st) return st;
  k1::Params p;
  memset(&p, 0, sizeof(p));
  int ih = 1, jw = 128;
  choose_tile_k1(g.rows, g.cols, ih, jw);
  const uint64_t cp = row_pitch(g.cols);
  {
    const uint64_t dims[4] = {128, (uint64_t)g.cols, (uint64_t)g.rows, (uint64_t)g.B};
    const uint64_t str[3] = {2ull * g.sc, 2ull * g.sr, 2ull * g.sb};
    const uint32_t box[4] = {64, (uint32_t)jw, (uint32_t)ih, 1};
    if ((st = encode_map(&p.tm_z, z, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[2] = {128, 512};
    const uint64_t str[1] = {256};
    const uint32_t box[2] = {64, 128};
    if ((st = encode_map(&p.tm_w, w->w_proj, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)g.cols, (uint64_t)g.rows, (uint64_t)g.B * 128};
    const uint64_t str[2] = {cp * 2, cp * 2 * g.rows};
    // one epilogue store: 32 positions x 32 channels, staged with the swizzle matching its row width
    const uint32_t w32 = jw < k1::SPOS ? jw : k1::SPOS;
    const uint32_t box[3] = {w32, k1::SPOS / w32, 32};
    const CUtensorMapSwizzle sw = w32 == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : w32 == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
    if ((st = encode_map(&p.tm_a, a, 3, dims, str, box, sw))) return st;
    if ((st = encode_map(&p.tm_b, b, 3, dims, str, box, sw))) return st;
  }
  p.ln_w = static_cast<const __half*>(w->ln_in_w);
  p.ln_b = static_cast<const __half*>(w->ln_in_b);
  p.bias = w->b_proj;
  p.mask = static_cast<const __half*>(mask);
  p.mask_sb = g.msb;
  p.mask_si = g.msr;
  p.mask_sj = g.msc;
  p.rows = g.rows;
  p.cols = g.cols;
  p.ih = ih;
  p.jw = jw;
  p.log2_jw = 31 - __builtin_clz(static_cast<unsigned>(jw));
  p.tiles_i = (g.rows + ih - 1) / ih;
  p.tiles_j = (g.cols + jw - 1) / jw;
  p.num_tiles = g.B * p.tiles_i * p.tiles_j;
  p.reset_status = reset_status ? 1 : 0;
  p.status = status;
  p.timeout_ns = g_timeout_ns;
  const int grid = std::min(p.num_tiles, dev.sms);
  cudaError_t e = launch_pdl(kern, grid, k1::kThreads, k1::SMEM_BYTES, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch project_gate_kernel");
}

// x[d] (M x N) = A[d] B[d]^T with K-deep rows.  K-major (outgoing form): a is [Bc, M, pitch(K)];
// b is `parts` consecutive blocks [Bc, rows_per_part, pitch(K)] (N = parts * rows_per_part), the
// layout an all-gather of row slabs produces.  MN-major (incoming form): a, b are [Bc, K, pitch(M)]
// with M = N = K (square only).  x is [Bc, M, pitch(N)].
template <int BN, bool MN>
int launch_k2_t(const void* a, const void* b, void* x, int Bc, int M, int N, int K, int rows_per_part, int ldx,
                DeviceStatus* status, cudaStream_t stream, unsigned attr_bit, int max_ctas) {
  using C = k2::Cfg<BN>;
  auto kern = &k2::contract_kernel<BN, MN>;
  Dev dev;
  int st = current_device(dev, attr_bit, reinterpret_cast<const void*>(kern), C::SMEM_BYTES);
  if (st) return st;
  k2::Params p;
  memset(&p, 0, sizeof(p));
  const uint64_t kp = row_pitch(K), np = ldx > 0 ? ldx : row_pitch(N);
  if (!MN) {
    const int parts = N / rows_per_part;
    const uint64_t da[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)Bc};
    const uint64_t sa[2] = {kp * 2, kp * 2 * M};
    const uint32_t boxa[3] = {64, 128, 1};
    if ((st = encode_map(&p.tm_a, a, 3, da, sa, boxa, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    const uint64_t db[4] = {(uint64_t)K, (uint64_t)rows_per_part, (uint64_t)Bc, (uint64_t)parts};
    const uint64_t sb[3] = {kp * 2, kp * 2 * rows_per_part, kp * 2 * rows_per_part * Bc};
    const uint32_t boxb[4] = {64, (uint32_t)BN, 1, 1};
    if ((st = encode_map(&p.tm_b, b, 4, db, sb, boxb, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  } else {
    const uint64_t dims[3] = {(uint64_t)M, (uint64_t)K, (uint64_t)Bc};
    const uint64_t str[2] = {row_pitch(M) * 2ull, row_pitch(M) * 2ull * K};
    const uint32_t box[3] = {64, 64, 1};
    if ((st = encode_map(&p.tm_a, a, 3, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    if ((st = encode_map(&p.tm_b, b, 3, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)Bc};
    const uint64_t str[2] = {np * 2, np * 2 * M};
    const uint32_t box[3] = {64, 128, 1};
    if ((st = encode_map(&p.tm_x, x, 3, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  p.N = N;
  p.rows_per_part = rows_per_part;
  p.tiles_m = (M + k2::BM - 1) / k2::BM;
  p.tiles_n = (N + BN - 1) / BN;
  p.num_tiles = Bc * p.tiles_m * p.tiles_n;
  p.num_kb = (K + k2::BK - 1) / k2::BK;
  p.status = status;
  p.timeout_ns = g_timeout_ns;
  int grid = std::min(p.num_tiles, dev.sms);
  if (max_ctas > 0) grid = std::min(grid, max_ctas);
  cudaError_t e = launch_pdl(kern, grid, k2::kThreads, C::SMEM_BYTES, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch contract_kernel");
}

// ldx: row pitch of x in elements (0: row_pitch(N)); x may be a column block of a wider matrix.
// max_ctas > 0 caps the persistent grid (leaving SMs to kernels that run alongside, e.g. NCCL's).
// The tile width for N columns: the least padding ceil(N / BN) * BN over BN in {128, 192, 256},
// ties to the wider tile (fewer tiles).
int choose_bn_k2(int N) {
  int best = 256;
  long long pad = static_cast<long long>((N + 255) / 256) * 256;
  for (int bn : {192, 128}) {
    const long long pb = static_cast<long long>((N + bn - 1) / bn) * bn;
    if (pb < pad) {
      pad = pb;
      best = bn;
    }
  }
  return best;
}

int launch_k2(const void* a, const void* b, void* x, int Bc, int M, int N, int K, int rows_per_part, bool outgoing,
              DeviceStatus* status, cudaStream_t stream, int ldx = 0, int max_ctas = 0) {
  const int bn = choose_bn_k2(N);
  if (!outgoing) {
    if (M != N || M != K || rows_per_part != N) return fail(TMU_ERR_UNSUPPORTED, "incoming form is square only");
    return bn == 128 ? launch_k2_t<128, true>(a, b, x, Bc, M, N, K, N, ldx, status, stream, 1u << 2, max_ctas)
         : bn == 192 ? launch_k2_t<192, true>(a, b, x, Bc, M, N, K, N, ldx, status, stream, 1u << 6, max_ctas)
                     : launch_k2_t<256, true>(a, b, x, Bc, M, N, K, N, ldx, status, stream, 1u << 4, max_ctas);
  }
  const int parts = N / rows_per_part;
  if (parts * rows_per_part != N) return fail(TMU_ERR_INVALID_ARGUMENT, "N must be a multiple of rows_per_part");
  if (parts == 1) {
    return bn == 128 ? launch_k2_t<128, false>(a, b, x, Bc, M, N, K, N, ldx, status, stream, 1u << 1, max_ctas)
         : bn == 192 ? launch_k2_t<192, false>(a, b, x, Bc, M, N, K, N, ldx, status, stream, 1u << 5, max_ctas)
                     : launch_k2_t<256, false>(a, b, x, Bc, M, N, K, N, ldx, status, stream, 1u << 3, max_ctas);
  }
  // a gathered B operand: a tile of BN rows must not straddle two parts
  if (rows_per_part % 256 == 0) return launch_k2_t<256, false>(a, b, x, Bc, M, N, K, rows_per_part, ldx, status, stream, 1u << 3, max_ctas);
  if (rows_per_part % 128 == 0) return launch_k2_t<128, false>(a, b, x, Bc, M, N, K, rows_per_part, ldx, status, stream, 1u << 1, max_ctas);
  return fail(TMU_ERR_UNSUPPORTED, "rows_per_part of a gathered operand must be a multiple of 128");
}

int launch_k3p(const void* x, const void* z, void* z_out, const tmu_trimul_weights* w, int B, int rows, int cols,
               float mix_eps, DeviceStatus* status, cudaStream_t stream);

int launch_k3(const void* x, const void* z, void* z_out, const tmu_trimul_weights* w, int B, int rows, int cols,
              float mix_eps, DeviceStatus* status, cudaStream_t stream, int cz) {
  // the emit and gate biases come together (both present, or neither: the reference's form)
  if ((w->b_emit == nullptr) != (w->b_gate == nullptr))
    return fail(TMU_ERR_INVALID_ARGUMENT, "b_emit and b_gate must both be set or both be NULL");
  if (cz == 256) return launch_k3p(x, z, z_out, w, B, rows, cols, mix_eps, status, stream);
  const bool hb = w->b_emit != nullptr;
  int ih = 1, jw = 128;
  choose_tile_k3(rows, cols, ih, jw);
  // jw >= 64: the x tile is loaded as two 128B-swizzled halves of 64 positions (one 128-byte
  // row per channel each), jw == 32 as four 64B-swizzled quarters (64-byte rows), and
  // transposed by ldmatrix.  (A box whose inner rows are shorter than the swizzle span cannot
  // take this form: TMA pads every such row to the span in shared memory, which would
  // quadruple the x tile's footprint at jw = 16 with the 128-byte swizzle.)
  const int xmode = jw >= 64 ? 1 : jw == 32 ? 2 : 0;
  void (*kern)(k3::Params) =
      hb ? (xmode == 1 ? k3::emit_residual_kernel<true, 1> : xmode == 2 ? k3::emit_residual_kernel<true, 2>
                                                                        : k3::emit_residual_kernel<true, 0>)
         : (xmode == 1 ? k3::emit_residual_kernel<false, 1> : xmode == 2 ? k3::emit_residual_kernel<false, 2>
                                                                         : k3::emit_residual_kernel<false, 0>);
  Dev dev;
  int st = current_device(dev, 1ull << ((xmode == 1 ? 40 : xmode == 2 ? 44 : 12) + (hb ? 1 : 0)),
                          reinterpret_cast<const void*>(kern), k3::SMEM_BYTES);
  if (st) return st;
  k3::Params p;
  memset(&p, 0, sizeof(p));
  const uint64_t cp = row_pitch(cols);
  {
    const uint64_t dims[4] = {128, (uint64_t)cols, (uint64_t)rows, (uint64_t)B};
    const uint64_t str[3] = {256, 256ull * cols, 256ull * cols * rows};
    const uint32_t box[4] = {64, (uint32_t)jw, (uint32_t)ih, 1};
    if ((st = encode_map(&p.tm_z, z, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    const uint32_t jwp = jw < 32 ? jw : 32;  // one epilogue warp's 32 positions
    const uint32_t boxo[4] = {64, jwp, 32 / jwp, 1};
    if ((st = encode_map(&p.tm_zo, z_out, 4, dims, str, boxo, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)cols, (uint64_t)rows, (uint64_t)B * 128};
    const uint64_t str[2] = {cp * 2, cp * 2 * rows};
    const uint32_t box[3] = {xmode == 1 ? 64u : (uint32_t)jw, xmode != 0 ? 1u : (uint32_t)ih, 128};
    const CUtensorMapSwizzle sw =
        xmode == 1 ? CU_TENSOR_MAP_SWIZZLE_128B : xmode == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE;
    if ((st = encode_map(&p.tm_x, x, 3, dims, str, box, sw))) return st;
  }
  {
    const uint64_t dims[2] = {128, 128};
    const uint64_t str[1] = {256};
    const uint32_t box[2] = {64, 128};
    if ((st = encode_map(&p.tm_we, w->w_emit, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    if ((st = encode_map(&p.tm_wg, w->w_gate, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  p.ln_in_w = static_cast<const __half*>(w->ln_in_w);
  p.ln_in_b = static_cast<const __half*>(w->ln_in_b);
  p.ln_mix_w = static_cast<const __half*>(w->ln_mix_w);
  p.ln_mix_b = static_cast<const __half*>(w->ln_mix_b);
  p.b_emit = w->b_emit;
  p.b_gate = w->b_gate;
  p.mix_eps = mix_eps;
  p.rows = rows;
  p.cols = cols;
  p.ih = ih;
  p.jw = jw;
  p.tiles_i = (rows + ih - 1) / ih;
  p.tiles_j = (cols + jw - 1) / jw;
  p.num_tiles = B * p.tiles_i * p.tiles_j;
  p.status = status;
  p.timeout_ns = g_timeout_ns;
  const int grid = std::min(p.num_tiles, dev.sms);
  cudaError_t e = launch_pdl(kern, grid, k3::kThreads, k3::SMEM_BYTES, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch emit_residual_kernel");
}

int g_pairs_k1p[kMaxDevices][8] = {{0}};

// K1 on CTA pairs (k1p_project.cuh), c_z = 128 or 256: tiles of 128 positions, shape chosen as
// K1's (the wide tiles from 512 x 512 positions up, the least padding below).  At c_z = 256 the
// pairs alternate between the operands a and b, so the pair count is even.
template <int CZ>
int launch_k1p(const void* z, const void* mask, const tmu_trimul_weights* w, const PairGeom& g, void* a, void* b,
               DeviceStatus* status, cudaStream_t stream, bool reset_status) {
  using C = k1p::Cfg<CZ>;
  const bool hb = w->b_proj != nullptr, hm = mask != nullptr;
  void (*kern)(k1p::Params) =
      hb ? (hm ? k1p::project_gate_pair_kernel<CZ, true, true> : k1p::project_gate_pair_kernel<CZ, true, false>)
         : (hm ? k1p::project_gate_pair_kernel<CZ, false, true> : k1p::project_gate_pair_kernel<CZ, false, false>);
  const int variant = (CZ == 256 ? 4 : 0) + (hb ? 2 : 0) + (hm ? 1 : 0);
  Dev dev;
  int st = current_device(dev, 1ull << (48 + variant), reinterpret_cast<const void*>(kern), C::SMEM_BYTES);
  if (st) return st;
  if (dev.sms < 4) return fail(TMU_ERR_UNSUPPORTED, "fewer than 4 SMs");
  int& pairs = g_pairs_k1p[dev.id][variant];
  if (pairs == 0) {
    pairs = max_resident_pairs(kern, k1p::kThreads, C::SMEM_BYTES);
    if (pairs == 0) pairs = dev.sms / 2;
  }
  k1p::Params p;
  memset(&p, 0, sizeof(p));
  int ih = 1, jw = 128;
  choose_tile_k1(g.rows, g.cols, ih, jw);
  const uint64_t cp = row_pitch(g.cols);
  {
    const uint64_t dims[4] = {(uint64_t)CZ, (uint64_t)g.cols, (uint64_t)g.rows, (uint64_t)g.B};
    const uint64_t str[3] = {2ull * g.sc, 2ull * g.sr, 2ull * g.sb};
    // a CTA's piece: rows [ih/2 r, ..) of the tile, or (ih = 1) columns [64 r, 64 r + 64)
    const uint32_t box[4] = {64, ih >= 2 ? (uint32_t)jw : 64u, ih >= 2 ? (uint32_t)(ih / 2) : 1u, 1};
    if ((st = encode_map(&p.tm_z, z, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)CZ, 4ull * CZ};
    const uint64_t str[1] = {2ull * CZ};
    const uint32_t box[2] = {64, 128};
    if ((st = encode_map(&p.tm_w, w->w_proj, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)g.cols, (uint64_t)g.rows, (uint64_t)g.B * CZ};
    const uint64_t str[2] = {cp * 2, cp * 2 * g.rows};
    const uint32_t w32 = jw < k1p::SPOS ? jw : k1p::SPOS;
    const uint32_t box[3] = {w32, k1p::SPOS / w32, 32};
    const CUtensorMapSwizzle sw = w32 == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : w32 == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
    if ((st = encode_map(&p.tm_a, a, 3, dims, str, box, sw))) return st;
    if ((st = encode_map(&p.tm_b, b, 3, dims, str, box, sw))) return st;
  }
  p.ln_w = static_cast<const __half*>(w->ln_in_w);
  p.ln_b = static_cast<const __half*>(w->ln_in_b);
  p.bias = w->b_proj;
  p.mask = static_cast<const __half*>(mask);
  p.mask_sb = g.msb;
  p.mask_si = g.msr;
  p.mask_sj = g.msc;
  p.rows = g.rows;
  p.cols = g.cols;
  p.ih = ih;
  p.jw = jw;
  p.log2_jw = 31 - __builtin_clz(static_cast<unsigned>(jw));
  p.tiles_i = (g.rows + ih - 1) / ih;
  p.tiles_j = (g.cols + jw - 1) / jw;
  p.num_tiles = (CZ == 256 ? 2 : 1) * g.B * p.tiles_i * p.tiles_j;
  p.reset_status = reset_status ? 1 : 0;
  p.status = status;
  p.timeout_ns = g_timeout_ns;
  // c_z = 256: an even pair count, so that a pair keeps one operand
  const int npairs = std::min(p.num_tiles, CZ == 256 ? (pairs & ~1) : pairs);
  cudaError_t e = launch_pdl_pair(kern, 2 * npairs, k1p::kThreads, C::SMEM_BYTES, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch project_gate_pair_kernel");
}

int g_pairs_k3p[kMaxDevices][2] = {{0}};

// K3 at c_z = 256 on CTA pairs (k3p_emit.cuh): tiles of 64 positions, 2 x 32 or 1 x 64, whichever
// pads less (the pair's CTAs take one row of 32 positions each).
int launch_k3p(const void* x, const void* z, void* z_out, const tmu_trimul_weights* w, int B, int rows, int cols,
               float mix_eps, DeviceStatus* status, cudaStream_t stream) {
  const uintptr_t bytes = static_cast<uintptr_t>(B) * rows * cols * 256 * 2;
  const uintptr_t zi = reinterpret_cast<uintptr_t>(z), zo = reinterpret_cast<uintptr_t>(z_out);
  if (zi < zo + bytes && zo < zi + bytes)
    return fail(TMU_ERR_INVALID_ARGUMENT, "c_z = 256: z_out must not overlap z (two CTAs share each tile's z)");
  const bool hb = w->b_emit != nullptr;
  const long long area2 = static_cast<long long>((rows + 1) / 2) * 2 * ((cols + 31) / 32) * 32;
  const long long area1 = static_cast<long long>(rows) * ((cols + 63) / 64) * 64;
  const int ih = area2 <= area1 ? 2 : 1, jw = 64 / ih;
  void (*kern)(k3p::Params) = hb ? k3p::emit_residual_pair_kernel<true> : k3p::emit_residual_pair_kernel<false>;
  Dev dev;
  int st = current_device(dev, 1ull << (46 + (hb ? 1 : 0)), reinterpret_cast<const void*>(kern), k3p::SMEM_BYTES);
  if (st) return st;
  if (dev.sms < 2) return fail(TMU_ERR_UNSUPPORTED, "fewer than 2 SMs");
  int& pairs = g_pairs_k3p[dev.id][hb ? 1 : 0];
  if (pairs == 0) {
    pairs = max_resident_pairs(kern, k3p::kThreads, k3p::SMEM_BYTES);
    if (pairs == 0) pairs = dev.sms / 2;
  }
  k3p::Params p;
  memset(&p, 0, sizeof(p));
  const uint64_t cp = row_pitch(cols);
  {
    const uint64_t dims[4] = {256, (uint64_t)cols, (uint64_t)rows, (uint64_t)B};
    const uint64_t str[3] = {512, 512ull * cols, 512ull * cols * rows};
    const uint32_t boxp[4] = {64, 32, 1, 1};
    if ((st = encode_map(&p.tm_z, z, 4, dims, str, boxp, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    const uint32_t boxt[4] = {64, (uint32_t)jw, (uint32_t)ih, 1};
    if ((st = encode_map(&p.tm_r, z, 4, dims, str, boxt, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    if ((st = encode_map(&p.tm_zo, z_out, 4, dims, str, boxt, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)cols, (uint64_t)rows, (uint64_t)B * 256};
    const uint64_t str[2] = {cp * 2, cp * 2 * rows};
    const uint32_t box[3] = {32, 1, 256};
    if ((st = encode_map(&p.tm_x, x, 3, dims, str, box, CU_TENSOR_MAP_SWIZZLE_64B))) return st;
  }
  p.w_emit = static_cast<const __half*>(w->w_emit);
  p.w_gate = static_cast<const __half*>(w->w_gate);
  p.ln_in_w = static_cast<const __half*>(w->ln_in_w);
  p.ln_in_b = static_cast<const __half*>(w->ln_in_b);
  p.ln_mix_w = static_cast<const __half*>(w->ln_mix_w);
  p.ln_mix_b = static_cast<const __half*>(w->ln_mix_b);
  p.b_emit = w->b_emit;
  p.b_gate = w->b_gate;
  p.mix_eps = mix_eps;
  p.rows = rows;
  p.cols = cols;
  p.ih = ih;
  p.jw = jw;
  p.tiles_i = (rows + ih - 1) / ih;
  p.tiles_j = (cols + jw - 1) / jw;
  p.num_tiles = B * p.tiles_i * p.tiles_j;
  p.status = status;
  p.timeout_ns = g_timeout_ns;
  const int grid = 2 * std::min(p.num_tiles, pairs);
  cudaError_t e = launch_pdl_pair(kern, grid, k3p::kThreads, k3p::SMEM_BYTES, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch emit_residual_pair_kernel");
}

template <int CZ>
int launch_k4(const void* z, void* z_out, const tmu_transition_weights* w, int B, int L, int hidden, bool swiglu,
              DeviceStatus* status, cudaStream_t stream) {
  void (*kern)(k4::Params) = swiglu ? k4::transition_kernel<CZ, true> : k4::transition_kernel<CZ, false>;
  constexpr int smem = k4::Cfg<CZ>::SMEM_BYTES;
  Dev dev;
  int st = current_device(dev, 1u << ((CZ == 256 ? 28 : 24) + (swiglu ? 1 : 0)), reinterpret_cast<const void*>(kern),
                          smem);
  if (st) return st;
  k4::Params p;
  memset(&p, 0, sizeof(p));
  int ih = 1, jw = 128;
  choose_tile(L, L, ih, jw, k4::TILE);
  {
    const uint64_t dims[4] = {CZ, (uint64_t)L, (uint64_t)L, (uint64_t)B};
    const uint64_t str[3] = {2ull * CZ, 2ull * CZ * L, 2ull * CZ * L * L};
    const uint32_t box[4] = {64, (uint32_t)jw, (uint32_t)ih, 1};
    if ((st = encode_map(&p.tm_z, z, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    const uint32_t jwp = jw < 32 ? jw : 32;  // one epilogue warp's 32 positions
    const uint32_t boxo[4] = {64, jwp, 32 / jwp, 1};
    if ((st = encode_map(&p.tm_zo, z_out, 4, dims, str, boxo, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[2] = {CZ, (uint64_t)(swiglu ? 2 * hidden : hidden)};
    const uint64_t str[1] = {2 * CZ};
    const uint32_t box[2] = {64, 64};
    if ((st = encode_map(&p.tm_w12, w->w12, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)hidden, CZ};
    const uint64_t str[1] = {2ull * hidden};
    const uint32_t box[2] = {64, 128};
    if ((st = encode_map(&p.tm_w3, w->w3, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  p.ln_w = static_cast<const __half*>(w->ln_w);
  p.ln_b = static_cast<const __half*>(w->ln_b);
  p.hidden = hidden;
  // SwiGLU chunks are 64 hidden units, ReLU chunks 128 (a last chunk past h reads zero rows
  // and zero w3 columns, which add exact zeros)
  p.nchunk = swiglu ? hidden / k4::CHUNK : (hidden + 2 * k4::CHUNK - 1) / (2 * k4::CHUNK);
  p.L = L;
  p.ih = ih;
  p.jw = jw;
  p.tiles_i = (L + ih - 1) / ih;
  p.tiles_j = (L + jw - 1) / jw;
  p.num_tiles = B * p.tiles_i * p.tiles_j;
  p.status = status;
  p.timeout_ns = g_timeout_ns;
  const int grid = std::min(p.num_tiles, dev.sms);
  cudaError_t e = launch_pdl(kern, grid, k4::kThreads, smem, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch transition_kernel");
}

// Row LayerNorm pass: h = fp16(LN(rows)) [rows, K].
template <int K, int SRC, int OUT = lnr::kOutF16>
int launch_lnr(const void* x1, const void* x2, int ld1, int ld2, const RowTerms* terms, const float* g,
               const float* b, void* out, long long rows, cudaStream_t stream) {
  void (*kern)(lnr::Params) = lnr::ln_rows_kernel<K, SRC, OUT>;
  Dev dev;
  int st = current_device(dev, 0, reinterpret_cast<const void*>(kern), 0);
  if (st) return st;
  lnr::Params p;
  memset(&p, 0, sizeof(p));
  p.x1 = x1;
  p.x2 = x2;
  p.ld1 = ld1;
  p.ld2 = ld2;
  if (terms) p.terms = *terms;
  p.g = g;
  p.b = b;
  p.out = out;
  p.rows = rows;
  p.eps = 1e-5f;
  constexpr int rows_per_cta = (lnr::kThreads / 32) * (K <= 256 ? 4 : 2);
  const long long need = (rows + rows_per_cta - 1) / rows_per_cta;
  const int grid = static_cast<int>(std::min<long long>(need, 8LL * dev.sms));
  cudaError_t e = launch_pdl(kern, grid, lnr::kThreads, 0, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch ln_rows_kernel");
}

// K4 in h mode: h = fp16(LN(z)) [B, L, L, CZ] by TMA, t = fp16(ffn) out, SwiGLU.
template <int CZ>
int launch_k4_h(const __half* h, __half* tout, const tmu_cond_transition_weights* w, int B, int L, int hidden,
                unsigned long long bit, DeviceStatus* status, cudaStream_t stream) {
  constexpr int MODE = k4::kModeH;
  void (*kern)(k4::Params) = k4::transition_kernel<CZ, true, MODE>;
  constexpr int smem = k4::Cfg<CZ, MODE>::SMEM_BYTES;
  Dev dev;
  int st = current_device(dev, bit, reinterpret_cast<const void*>(kern), smem);
  if (st) return st;
  k4::Params p;
  memset(&p, 0, sizeof(p));
  int ih = 1, jw = 128;
  choose_tile(L, L, ih, jw, k4::TILE);
  {
    const uint64_t dims[4] = {CZ, (uint64_t)L, (uint64_t)L, (uint64_t)B};
    const uint64_t str[3] = {2ull * CZ, 2ull * CZ * L, 2ull * CZ * L * L};
    const uint32_t box[4] = {64, (uint32_t)jw, (uint32_t)ih, 1};
    if ((st = encode_map(&p.tm_z, h, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[2] = {CZ, (uint64_t)(2 * hidden)};
    const uint64_t str[1] = {2 * CZ};
    const uint32_t box[2] = {64, 64};
    if ((st = encode_map(&p.tm_w12, w->w12, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)hidden, CZ};
    const uint64_t str[1] = {2ull * hidden};
    const uint32_t box[2] = {64, 128};
    if ((st = encode_map(&p.tm_w3, w->w3, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  p.tout = tout;
  p.hidden = hidden;
  p.nchunk = hidden / k4::CHUNK;
  p.L = L;
  p.ih = ih;
  p.jw = jw;
  p.tiles_i = (L + ih - 1) / ih;
  p.tiles_j = (L + jw - 1) / jw;
  p.num_tiles = B * p.tiles_i * p.tiles_j;
  p.status = status;
  p.timeout_ns = g_timeout_ns;
  const int grid = std::min(p.num_tiles, dev.sms);
  cudaError_t e = launch_pdl(kern, grid, k4::kThreads, smem, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch transition_kernel (h)");
}

// K6 with the A operand by TMA: D = h @ W^T over a K-step schedule (step s: A channels
// [a_coord[s], +64) of the ka-wide h rows times W columns [w_coord[s], +64) of the kw-wide W rows).
struct K6Sched {
  int nsteps;
  short a_coord[k6::kMaxSteps];
  short w_coord[k6::kMaxSteps];
};

K6Sched plain_sched(int K) {
  K6Sched sc;
  sc.nsteps = K / 64;
  for (int k = 0; k < sc.nsteps; ++k) sc.a_coord[k] = sc.w_coord[k] = static_cast<short>(64 * k);
  return sc;
}

template <int EPI, bool BF16 = false>
int launch_k6g(const void* h, int ka, const void* w, int kw, int n, const K6Sched& sc, void* out, const void* bias,
               int heads, const float* zres, const float* avec, int B, int L, unsigned long long bit,
               DeviceStatus* status, cudaStream_t stream) {
  void (*kern)(k6::Params) = k6::gemm_kernel<EPI, BF16>;
  Dev dev;
  int st = current_device(dev, bit, reinterpret_cast<const void*>(kern), k6::SMEM_BYTES);
  if (st) return st;
  k6::Params p;
  memset(&p, 0, sizeof(p));
  int ih = 1, jw = 128;
  choose_tile(L, L, ih, jw, k6::TILE);
  {
    const uint64_t dims[2] = {(uint64_t)kw, (uint64_t)n};
    const uint64_t str[1] = {2ull * kw};
    const uint32_t box[2] = {64, (uint32_t)n};
    if ((st = encode_map(&p.tm_w, w, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[4] = {(uint64_t)ka, (uint64_t)L, (uint64_t)L, (uint64_t)B};
    const uint64_t str[3] = {2ull * ka, 2ull * ka * L, 2ull * ka * L * L};
    const uint32_t box[4] = {64, (uint32_t)jw, (uint32_t)ih, 1};
    if ((st = encode_map(&p.tm_a, h, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  p.out = out;
  p.bias = static_cast<const __half*>(bias);
  p.zres = zres;
  p.avec = avec;
  p.n = n;
  p.heads = heads;
  p.nsteps = sc.nsteps;
  for (int k = 0; k < sc.nsteps; ++k) {
    p.a_coord[k] = sc.a_coord[k];
    p.w_coord[k] = sc.w_coord[k];
  }
  p.B = B;
  p.L = L;
  p.ih = ih;
  p.jw = jw;
  p.tiles_i = (L + ih - 1) / ih;
  p.tiles_j = (L + jw - 1) / jw;
  p.num_tiles = B * p.tiles_i * p.tiles_j;
  p.status = status;
  p.timeout_ns = g_timeout_ns;
  const int grid = std::min(p.num_tiles, dev.sms);
  cudaError_t e = launch_pdl(kern, grid, k6::kThreads, k6::SMEM_BYTES, stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch gemm_kernel");
}

template <int CZ>
int launch_k5(const void* z, const void* w, const float* bias, const float* centres, float* out, int B, int L,
              DeviceStatus* status, cudaStream_t stream) {
  using C = k5::Cfg<CZ>;
  auto kern = &k5::disto_kernel<CZ>;
  Dev dev;
  int st = current_device(dev, 1u << (26 + (CZ == 256 ? 1 : 0)), reinterpret_cast<const void*>(kern), C::SMEM_BYTES);
  if (st) return st;
  k5::Params p;
  memset(&p, 0, sizeof(p));
  int ih = 1, jw = 128;
  choose_tile(L, L, ih, jw, k5::TILE);
  const uint64_t e = 2ull * CZ;  // bytes per position
  {
    const uint64_t dims[4] = {(uint64_t)CZ, (uint64_t)L, (uint64_t)L, (uint64_t)B};
    const uint32_t box[4] = {64, (uint32_t)jw, (uint32_t)ih, 1};
    const uint64_t str[3] = {e, e * L, e * L * L};     // (c, j, i, b) -> z[b, i, j, c]
    if ((st = encode_map(&p.tm_z, z, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    const uint64_t strt[3] = {e * L, e, e * L * L};    // (c, j, i, b) -> z[b, j, i, c]
    if ((st = encode_map(&p.tm_zt, z, 4, dims, strt, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)CZ, (uint64_t)k5::NBINS};
    const uint64_t str[1] = {e};
    const uint32_t box[2] = {64, 128};
    if ((st = encode_map(&p.tm_w, w, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  p.bias = bias;
  p.centres = centres;
  p.out = out;
  p.L = L;
  p.ih = ih;
  p.jw = jw;
  p.tiles_i = (L + ih - 1) / ih;
  p.tiles_j = (L + jw - 1) / jw;
  p.num_tiles = B * p.tiles_i * p.tiles_j;
  p.status = status;
  p.timeout_ns = g_timeout_ns;
  const int grid = std::min(p.num_tiles, dev.sms);
  cudaError_t err = launch_pdl(kern, grid, k5::kThreads, C::SMEM_BYTES, stream, p);
  if (err == cudaSuccess) err = cudaGetLastError();
  return err == cudaSuccess ? TMU_OK : cuda_fail(err, "launch disto_kernel");
}

size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

size_t cm_bytes(int B, int L, int c) { return align256(static_cast<size_t>(B) * c * L * row_pitch(L) * 2); }

__global__ void wait_timeout_kernel(DeviceStatus* status, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ volatile int abort_sh;
  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const WaitCtx ctx{status, &abort_sh, timeout_ns};
    mbar_wait(&bar, 0, ctx, 0x901u);  // nothing arrives: must give up and record the timeout
  }
}

// ------------------------------------------------------------------------------------------
// Scratch for tmu_trimul_noalloc: a fixed, statically sized device array, so that entry point
// never allocates.  It lives in this library's module on every GPU that loads the library, for
// the life of the process.  Host code must not hand the symbol itself to a kernel (on the host it
// is only a stand-in); the device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, and cached.
// ------------------------------------------------------------------------------------------
constexpr size_t kNoAllocBufBytes = TMU_NOALLOC_MAX_BUFFER_BYTES;
constexpr size_t kNoAllocBytes = TMU_STATUS_BYTES + 3 * kNoAllocBufBytes;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];
void* g_noalloc_addr[kMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

int noalloc_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(TMU_ERR_INVALID_ARGUMENT, "device id out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return TMU_OK;
}

}  // namespace

extern "C" {

const char* tmu_version(void) { return "tmu-b200 0.1 (sm_100a)"; }

const char* tmu_status_name(int s) {
  switch (s) {
    case TMU_OK: return "TMU_OK";
    case TMU_ERR_INVALID_ARGUMENT: return "TMU_ERR_INVALID_ARGUMENT";
    case TMU_ERR_MISALIGNED: return "TMU_ERR_MISALIGNED";
    case TMU_ERR_WORKSPACE_TOO_SMALL: return "TMU_ERR_WORKSPACE_TOO_SMALL";
    case TMU_ERR_UNSUPPORTED: return "TMU_ERR_UNSUPPORTED";
    case TMU_ERR_CUDA: return "TMU_ERR_CUDA";
    case TMU_ERR_DEVICE_TIMEOUT: return "TMU_ERR_DEVICE_TIMEOUT";
    case TMU_ERR_ARCH: return "TMU_ERR_ARCH";
    case TMU_ERR_DRIVER: return "TMU_ERR_DRIVER";
    case TMU_ERR_SMEM_LAYOUT: return "TMU_ERR_SMEM_LAYOUT";
    default: return "TMU_ERR_UNKNOWN";
  }
}

const char* tmu_last_error(void) { return g_last_error.c_str(); }

int tmu_device_check(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    char buf[96];
    snprintf(buf, sizeof(buf), "device %d is sm_%d%d; kernels are built for sm_100a", dev, major, minor);
    return fail(TMU_ERR_ARCH, buf);
  }
  return TMU_OK;
}

int tmu_row_pitch(int L) { return row_pitch(L); }

int tmu_proj_row_order(int c, int* order) {
  if (order == nullptr || c <= 0 || c % 64 != 0) return fail(TMU_ERR_INVALID_ARGUMENT, "c must be a multiple of 64");
  // blocks of c rows: [signal a | gate a | signal b | gate b]; proj_bundle rows are
  // [signal a | signal b | gate a | gate b] (mlx_trunk.py:44)
  for (int r = 0; r < c; ++r) {
    order[r] = r;                // signal a
    order[c + r] = 2 * c + r;    // gate a
    order[2 * c + r] = c + r;    // signal b
    order[3 * c + r] = 3 * c + r;  // gate b
  }
  return TMU_OK;
}

size_t tmu_workspace_bytes(int B, int L, int c_z, int c) {
  (void)c_z;
  if (B < 1 || L < 1 || c < 1) return 0;
  return TMU_STATUS_BYTES + 3 * cm_bytes(B, L, c);
}

unsigned long long tmu_set_wait_timeout_ns(unsigned long long ns) {
  const unsigned long long old = g_timeout_ns;
  g_timeout_ns = ns;
  return old;
}

int tmu_reset_status(void* status, void* stream) {
  if (status == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "status is NULL");
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(DeviceStatus), static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "cudaMemsetAsync(status)");
}

int tmu_read_status(const void* status, void* stream, int* code, int* site) {
  if (status == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "status is NULL");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  DeviceStatus h;
  e = cudaMemcpy(&h, status, sizeof(h), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
  if (code) *code = static_cast<int>(h.code);
  if (site) *site = static_cast<int>(h.site);
  return TMU_OK;
}

int tmu_trace_arm(void* status, void* stream) {
  if (status == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "status is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* b = static_cast<uint8_t*>(status);
  cudaError_t e = cudaMemsetAsync(b, 0, sizeof(DeviceStatus), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(b + offsetof(DeviceStatus, trace_flag), 1, 1, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(b + offsetof(DeviceStatus, t_start), 0xff, sizeof(unsigned long long), s);
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "cudaMemsetAsync(trace)");
}

int tmu_trace_read(const void* status, void* stream, unsigned long long* t_start, unsigned long long* t_end) {
  if (status == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "status is NULL");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  DeviceStatus h;
  e = cudaMemcpy(&h, status, sizeof(h), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
  if (t_start) *t_start = h.t_start;
  if (t_end) *t_end = h.t_end;
  return TMU_OK;
}

int tmu_read_first_error(const void* status, void* stream, int* code, int* site) {
  if (status == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "status is NULL");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  DeviceStatus h;
  e = cudaMemcpy(&h, status, sizeof(h), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
  if (code) *code = static_cast<int>(h.first_code);
  if (site) *site = static_cast<int>(h.first_site);
  return TMU_OK;
}

int tmu_project_gate(const void* z, const void* mask, const tmu_trimul_weights* w, int B, int L, int c_z, int c,
                     void* a, void* b, void* status, void* stream) {
  int st = check_sizes(B, L, c_z, c);
  if (st) return st;
  if ((st = check_weights(w, true, false))) return st;
  if (!z || !a || !b || !status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (!aligned16(z) || !aligned16(a) || !aligned16(b)) return fail(TMU_ERR_MISALIGNED, "z/a/b not 16-byte aligned");
  return launch_k1(z, mask, w, square_geom(B, L, c_z), a, b, static_cast<DeviceStatus*>(status),
                   static_cast<cudaStream_t>(stream));
}

int tmu_contract(const void* a, const void* b, void* x, int Bc, int L, int outgoing, void* status, void* stream) {
  if (Bc < 1 || L < 1) return fail(TMU_ERR_INVALID_ARGUMENT, "Bc and L must be positive");
  if (L > 8192 || Bc > 65535) return fail(TMU_ERR_UNSUPPORTED, "L > 8192 or Bc > 65535");
  if (!a || !b || !x || !status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (!aligned16(a) || !aligned16(b) || !aligned16(x)) return fail(TMU_ERR_MISALIGNED, "a/b/x not 16-byte aligned");
  return launch_k2(a, b, x, Bc, L, L, L, L, outgoing != 0, static_cast<DeviceStatus*>(status),
                   static_cast<cudaStream_t>(stream));
}

int tmu_emit_residual(const void* x, const void* z, void* z_out, const tmu_trimul_weights* w, int B, int L, int c_z,
                      int c, float mix_eps, void* status, void* stream) {
  int st = check_sizes(B, L, c_z, c);
  if (st) return st;
  if ((st = check_weights(w, false, true))) return st;
  if (!x || !z || !z_out || !status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (!aligned16(x) || !aligned16(z) || !aligned16(z_out)) return fail(TMU_ERR_MISALIGNED, "x/z not 16-byte aligned");
  if (!(mix_eps > 0.f)) return fail(TMU_ERR_INVALID_ARGUMENT, "mix_eps must be positive");
  return launch_k3(x, z, z_out, w, B, L, L, mix_eps, static_cast<DeviceStatus*>(status),
                   static_cast<cudaStream_t>(stream), c_z);
}

int tmu_project_gate_ex(const void* z, const void* mask, const tmu_pair_layout* g, const tmu_trimul_weights* w,
                        int c_z, int c, void* a, void* b, void* status, void* stream) {
  if (g == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "layout is NULL");
  if (g->rows < 1 || g->cols < 1 || g->B < 1) return fail(TMU_ERR_INVALID_ARGUMENT, "empty pair grid");
  int st = check_sizes(g->B, std::max(g->rows, g->cols), c_z, c);
  if (st) return st;
  if ((st = check_weights(w, true, false))) return st;
  if (!z || !a || !b || !status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (!aligned16(z) || !aligned16(a) || !aligned16(b)) return fail(TMU_ERR_MISALIGNED, "z/a/b not 16-byte aligned");
  if (g->stride_col % 8 || g->stride_row % 8 || g->stride_b % 8)
    return fail(TMU_ERR_MISALIGNED, "z strides must be multiples of 8 elements (16 bytes)");
  const PairGeom pg{g->B, g->rows, g->cols, g->stride_b, g->stride_row, g->stride_col,
                    g->mask_stride_b, g->mask_stride_row, g->mask_stride_col, c_z};
  return launch_k1(z, mask, w, pg, a, b, static_cast<DeviceStatus*>(status), static_cast<cudaStream_t>(stream));
}

int tmu_contract_ex(const void* a, const void* b, void* x, int Bc, int M, int N, int K, int b_rows_per_part,
                    int ldx, int max_ctas, void* status, void* stream) {
  if (Bc < 1 || M < 1 || N < 1 || K < 1 || b_rows_per_part < 1)
    return fail(TMU_ERR_INVALID_ARGUMENT, "sizes must be positive");
  if (ldx != 0 && (ldx < N || ldx % 8 != 0))
    return fail(TMU_ERR_INVALID_ARGUMENT, "ldx must be 0 or a multiple of 8 that is >= N");
  if (M > 8192 || N > 8192 || K > 8192 || Bc > 65535) return fail(TMU_ERR_UNSUPPORTED, "size too large");
  if (!a || !b || !x || !status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (!aligned16(a) || !aligned16(b) || !aligned16(x)) return fail(TMU_ERR_MISALIGNED, "a/b/x not 16-byte aligned");
  if (max_ctas < 0) return fail(TMU_ERR_INVALID_ARGUMENT, "max_ctas must be >= 0");
  return launch_k2(a, b, x, Bc, M, N, K, b_rows_per_part, true, static_cast<DeviceStatus*>(status),
                   static_cast<cudaStream_t>(stream), ldx, max_ctas);
}

int tmu_emit_residual_ex(const void* x, const void* z, void* z_out, int B, int rows, int cols,
                         const tmu_trimul_weights* w, int c_z, int c, float mix_eps, void* status, void* stream) {
  if (rows < 1 || cols < 1) return fail(TMU_ERR_INVALID_ARGUMENT, "empty pair grid");
  int st = check_sizes(B, std::max(rows, cols), c_z, c);
  if (st) return st;
  if ((st = check_weights(w, false, true))) return st;
  if (!x || !z || !z_out || !status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (!aligned16(x) || !aligned16(z) || !aligned16(z_out)) return fail(TMU_ERR_MISALIGNED, "x/z not 16-byte aligned");
  if (!(mix_eps > 0.f)) return fail(TMU_ERR_INVALID_ARGUMENT, "mix_eps must be positive");
  return launch_k3(x, z, z_out, w, B, rows, cols, mix_eps, static_cast<DeviceStatus*>(status),
                   static_cast<cudaStream_t>(stream), c_z);
}

int tmu_trimul(const void* z, void* z_out, const void* mask, const tmu_trimul_weights* w, int B, int L, int c_z,
               int c, int outgoing, float mix_eps, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_sizes(B, L, c_z, c);
  if (st) return st;
  if ((st = check_weights(w, true, true))) return st;
  if (!z || !z_out || !workspace) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail(TMU_ERR_MISALIGNED, "workspace not 256-byte aligned");
  if (!aligned16(z) || !aligned16(z_out)) return fail(TMU_ERR_MISALIGNED, "z not 16-byte aligned");
  if (workspace_bytes < tmu_workspace_bytes(B, L, c_z, c)) return fail(TMU_ERR_WORKSPACE_TOO_SMALL, "workspace too small");
  if (!(mix_eps > 0.f)) return fail(TMU_ERR_INVALID_ARGUMENT, "mix_eps must be positive");
  if ((st = check_wide_alias(z, z_out, B, L, c_z))) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  DeviceStatus* status = reinterpret_cast<DeviceStatus*>(ws);
  const size_t cm = cm_bytes(B, L, c);
  void* a = ws + TMU_STATUS_BYTES;
  void* b = ws + TMU_STATUS_BYTES + cm;
  void* x = ws + TMU_STATUS_BYTES + 2 * cm;
  // K1 zeroes the status word after its dependency wait (no memset node between the kernels,
  // so the three launches chain with programmatic dependent launch)
  if ((st = launch_k1(z, mask, w, square_geom(B, L, c_z), a, b, status, s, true))) return st;
  if ((st = launch_k2(a, b, x, B * c, L, L, L, L, outgoing != 0, status, s))) return st;
  return launch_k3(x, z, z_out, w, B, L, L, mix_eps, status, s, c_z);
}

int tmu_trimul_noalloc(const void* z, void* z_out, const void* mask, const tmu_trimul_weights* w, int B, int L,
                       int c_z, int c, int outgoing, float mix_eps, void* status, void* stream) {
  int st = check_sizes(B, L, c_z, c);
  if (st) return st;
  if ((st = check_weights(w, true, true))) return st;
  if (!z || !z_out) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (!aligned16(z) || !aligned16(z_out)) return fail(TMU_ERR_MISALIGNED, "z not 16-byte aligned");
  if (status != nullptr && !aligned16(status)) return fail(TMU_ERR_MISALIGNED, "status not 16-byte aligned");
  if (!(mix_eps > 0.f)) return fail(TMU_ERR_INVALID_ARGUMENT, "mix_eps must be positive");
  if ((st = check_wide_alias(z, z_out, B, L, c_z))) return st;
  const size_t cm = cm_bytes(B, L, c);
  if (cm > kNoAllocBufBytes) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "tmu_trimul_noalloc: B*c*L*row_pitch(L)*2 = %zu bytes exceeds the static scratch of %zu bytes per "
             "buffer; use tmu_trimul with a caller-provided workspace",
             static_cast<size_t>(B) * c * L * row_pitch(L) * 2, kNoAllocBufBytes);
    return fail(TMU_ERR_UNSUPPORTED, buf);
  }
  void* scratch = nullptr;
  if ((st = noalloc_scratch_address(&scratch))) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  DeviceStatus* dstat = reinterpret_cast<DeviceStatus*>(status != nullptr ? status : base);
  void* a = base + TMU_STATUS_BYTES;
  void* b = base + TMU_STATUS_BYTES + kNoAllocBufBytes;
  void* x = base + TMU_STATUS_BYTES + 2 * kNoAllocBufBytes;
  // the status word must start at zero; a, b and x are fully rewritten before they are read
  if ((st = tmu_reset_status(dstat, stream))) return st;
  if ((st = launch_k1(z, mask, w, square_geom(B, L, c_z), a, b, dstat, s))) return st;
  if ((st = launch_k2(a, b, x, B * c, L, L, L, L, outgoing != 0, dstat, s))) return st;
  return launch_k3(x, z, z_out, w, B, L, L, mix_eps, dstat, s, c_z);
}

// Host-side checks of a transition call (shared by tmu_transition and tmu_pair_block).
static int check_transition(const void* z, const void* z_out, const tmu_transition_weights* w, int B, int L, int c_z,
                            int hidden, int activation) {
  if (B < 1 || L < 1) return fail(TMU_ERR_INVALID_ARGUMENT, "B and L must be positive");
  if (c_z != 128 && c_z != 256) return fail(TMU_ERR_UNSUPPORTED, "c_z must be 128 or 256");
  if (hidden < 64 || hidden > 4096 || hidden % 64) return fail(TMU_ERR_UNSUPPORTED, "hidden must be a multiple of 64 in [64, 4096]");
  if (L > 8192 || B > 65535) return fail(TMU_ERR_UNSUPPORTED, "L > 8192");
  if (activation != TMU_ACT_SWIGLU && activation != TMU_ACT_RELU) return fail(TMU_ERR_INVALID_ARGUMENT, "unknown activation");
  if (w == nullptr || !w->ln_w || !w->ln_b || !w->w12 || !w->w3) return fail(TMU_ERR_INVALID_ARGUMENT, "transition weights missing");
  if (!z || !z_out) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  const void* al[] = {z, z_out, w->ln_w, w->ln_b, w->w12, w->w3};
  for (const void* q : al)
    if (!aligned16(q)) return fail(TMU_ERR_MISALIGNED, "pointer not 16-byte aligned");
  return TMU_OK;
}

int tmu_transition(const void* z, void* z_out, const tmu_transition_weights* w, int B, int L, int c_z, int hidden,
                   int activation, void* status, void* stream) {
  int rc = check_transition(z, z_out, w, B, L, c_z, hidden, activation);
  if (rc) return rc;
  if (!status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  const bool swiglu = activation == TMU_ACT_SWIGLU;
  DeviceStatus* st = static_cast<DeviceStatus*>(status);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return c_z == 128 ? launch_k4<128>(z, z_out, w, B, L, hidden, swiglu, st, s)
                    : launch_k4<256>(z, z_out, w, B, L, hidden, swiglu, st, s);
}

size_t tmu_pair_block_workspace_bytes(int B, int L, int c_z, int c) {
  const size_t tm = tmu_workspace_bytes(B, L, c_z, c);
  if (tm == 0 || c_z < 1) return 0;
  const size_t pair = c_z == 256 ? (static_cast<size_t>(B) * L * L * c_z * 2 + 255) / 256 * 256 : 0;
  return tm + pair;
}

int tmu_pair_block(const void* z, void* z_out, const void* mask, const tmu_trimul_weights* w_out,
                   const tmu_trimul_weights* w_in, const tmu_transition_weights* w_tr, int B, int L, int c_z, int c,
                   int hidden, int activation, float mix_eps, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_sizes(B, L, c_z, c);
  if (st) return st;
  if ((st = check_weights(w_out, true, true))) return st;
  if ((st = check_weights(w_in, true, true))) return st;
  if ((st = check_transition(z, z_out, w_tr, B, L, c_z, hidden, activation))) return st;
  // checked here as well as in each launch, so that a bad argument launches nothing
  for (const tmu_trimul_weights* w : {w_out, w_in})
    if ((w->b_emit == nullptr) != (w->b_gate == nullptr))
      return fail(TMU_ERR_INVALID_ARGUMENT, "b_emit and b_gate must both be set or both be NULL");
  if (!workspace) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail(TMU_ERR_MISALIGNED, "workspace not 256-byte aligned");
  if (workspace_bytes < tmu_pair_block_workspace_bytes(B, L, c_z, c))
    return fail(TMU_ERR_WORKSPACE_TOO_SMALL, "workspace too small");
  if (!(mix_eps > 0.f)) return fail(TMU_ERR_INVALID_ARGUMENT, "mix_eps must be positive");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  DeviceStatus* status = reinterpret_cast<DeviceStatus*>(ws);
  const size_t cm = cm_bytes(B, L, c);
  void* a = ws + TMU_STATUS_BYTES;
  void* b = ws + TMU_STATUS_BYTES + cm;
  void* x = ws + TMU_STATUS_BYTES + 2 * cm;
  // c_z = 128 updates in place; the wide kernels write the outgoing result to the pair buffer
  void* mid = c_z == 256 ? static_cast<void*>(ws + tmu_workspace_bytes(B, L, c_z, c)) : z_out;
  const PairGeom g = square_geom(B, L, c_z);
  // the first kernel zeroes the shared status word; the six after it only record errors
  if ((st = launch_k1(z, mask, w_out, g, a, b, status, s, true))) return st;
  if ((st = launch_k2(a, b, x, B * c, L, L, L, L, true, status, s))) return st;
  if ((st = launch_k3(x, z, mid, w_out, B, L, L, mix_eps, status, s, c_z))) return st;
  if ((st = launch_k1(mid, mask, w_in, g, a, b, status, s))) return st;
  if ((st = launch_k2(a, b, x, B * c, L, L, L, L, false, status, s))) return st;
  if ((st = launch_k3(x, mid, z_out, w_in, B, L, L, mix_eps, status, s, c_z))) return st;
  const bool swiglu = activation == TMU_ACT_SWIGLU;
  return c_z == 128 ? launch_k4<128>(z_out, z_out, w_tr, B, L, hidden, swiglu, status, s)
                    : launch_k4<256>(z_out, z_out, w_tr, B, L, hidden, swiglu, status, s);
}

int tmu_disto_expected(const void* z, const void* w, const float* bias, const float* centres, float* out, int B,
                       int L, int c_z, int n_bins, void* status, void* stream) {
  if (B < 1 || L < 1) return fail(TMU_ERR_INVALID_ARGUMENT, "B and L must be positive");
  if (c_z != 128 && c_z != 256) return fail(TMU_ERR_UNSUPPORTED, "c_z must be 128 or 256");
  if (n_bins != k5::NBINS) return fail(TMU_ERR_UNSUPPORTED, "the distogram head must have 128 bins");
  if (L > 8192 || B > 65535) return fail(TMU_ERR_UNSUPPORTED, "L > 8192");
  if (!z || !w || !centres || !out || !status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (!aligned16(z) || !aligned16(w)) return fail(TMU_ERR_MISALIGNED, "z/w not 16-byte aligned");
  DeviceStatus* st = static_cast<DeviceStatus*>(status);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return c_z == 128 ? launch_k5<128>(z, w, bias, centres, out, B, L, st, s)
                    : launch_k5<256>(z, w, bias, centres, out, B, L, st, s);
}

namespace {
size_t pc_term_bytes(int B, int L, int c) { return (static_cast<size_t>(B) * L * L * c * 2 + 255) / 256 * 256; }
}  // namespace

size_t tmu_pair_cond_workspace_bytes(int B, int L, int c_in, int c_pair, int n_transitions) {
  if (B < 1 || L < 1 || c_in < 1 || c_pair < 1 || n_transitions < 0) return 0;
  return pc_term_bytes(B, L, c_pair) * (n_transitions + 1) + pc_term_bytes(B, L, std::max(c_in, c_pair));
}

int tmu_pair_cond(const float* z_trunk, const float* rel_pos, const tmu_pair_cond_weights* w, int B, int L,
                  int c_trunk, int c_rel, int c_pair, int hidden, int n_bias, int heads, void* out,
                  void* workspace, size_t workspace_bytes, void* status, void* stream) {
  if (B < 1 || L < 1) return fail(TMU_ERR_INVALID_ARGUMENT, "B and L must be positive");
  if (L > 8192 || B > 65535) return fail(TMU_ERR_UNSUPPORTED, "L > 8192");
  if (c_trunk != c_rel || (c_trunk + c_rel != 256 && c_trunk + c_rel != 512))
    return fail(TMU_ERR_UNSUPPORTED, "c_trunk == c_rel with c_trunk + c_rel = 256 or 512 is built");
  if (c_pair != 128 && c_pair != 256) return fail(TMU_ERR_UNSUPPORTED, "c_pair must be 128 or 256");
  if (w == nullptr || !w->ln_w || !w->ln_b || !w->proj || !w->bias_w || !w->bias_b ||
      w->n_transitions < 0 || (w->n_transitions > 0 && !w->transitions))
    return fail(TMU_ERR_INVALID_ARGUMENT, "pair conditioning weights missing");
  if (w->n_transitions > kMaxTerms - 1) return fail(TMU_ERR_UNSUPPORTED, "at most 3 transitions");
  if (w->n_transitions > 0 && (hidden < 64 || hidden > 4096 || hidden % 64))
    return fail(TMU_ERR_UNSUPPORTED, "hidden must be a multiple of 64 in [64, 4096]");
  if (n_bias < 16 || n_bias > 256 || n_bias % 16 || heads < 1 || n_bias % heads)
    return fail(TMU_ERR_UNSUPPORTED, "n_bias must be a multiple of 16 in [16, 256], divisible by heads");
  if (!z_trunk || !rel_pos || !out || !workspace || !status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  const int c_in = c_trunk + c_rel;
  if (workspace_bytes < tmu_pair_cond_workspace_bytes(B, L, c_in, c_pair, w->n_transitions))
    return fail(TMU_ERR_WORKSPACE_TOO_SMALL, "workspace too small");
  const void* al[] = {z_trunk, rel_pos, out, workspace, w->ln_w, w->ln_b, w->proj, w->bias_w};
  for (const void* q : al)
    if (!aligned16(q)) return fail(TMU_ERR_MISALIGNED, "pointer not 16-byte aligned");
  for (int t = 0; t < w->n_transitions; ++t) {
    const tmu_cond_transition_weights& tw = w->transitions[t];
    if (!tw.ln_w || !tw.ln_b || !tw.w12 || !tw.w3) return fail(TMU_ERR_INVALID_ARGUMENT, "transition weights missing");
    if (!aligned16(tw.ln_w) || !aligned16(tw.ln_b) || !aligned16(tw.w12) || !aligned16(tw.w3))
      return fail(TMU_ERR_MISALIGNED, "pointer not 16-byte aligned");
  }
  DeviceStatus* st = static_cast<DeviceStatus*>(status);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long cells = static_cast<long long>(B) * L * L;
  // Workspace: the fp32 residual stream as its fp16 terms (z0, then each transition's t_k), then
  // one h buffer for the LayerNorm pass in front of each GEMM kernel.
  const size_t term = pc_term_bytes(B, L, c_pair);
  RowTerms terms;
  memset(&terms, 0, sizeof(terms));
  terms.ld = c_pair;
  for (int k = 0; k <= w->n_transitions; ++k)
    terms.src[k] = reinterpret_cast<const __half*>(static_cast<uint8_t*>(workspace) + k * term);
  __half* z0 = static_cast<__half*>(workspace);
  __half* h = reinterpret_cast<__half*>(static_cast<uint8_t*>(workspace) + (w->n_transitions + 1) * term);
  const bool wide = c_pair == 256;
  // Stage A: h = fp16(LN(concat)), z0 = fp16(h @ proj^T)
  int r = c_in == 512 ? launch_lnr<512, kRowCat32>(z_trunk, rel_pos, c_trunk, c_rel, nullptr, w->ln_w, w->ln_b, h, cells, s)
                      : launch_lnr<256, kRowCat32>(z_trunk, rel_pos, c_trunk, c_rel, nullptr, w->ln_w, w->ln_b, h, cells, s);
  if (r) return r;
  r = launch_k6g<k6::kEpiStore16>(h, c_in, w->proj, c_in, c_pair, plain_sched(c_in), z0, nullptr, 1, nullptr, nullptr,
                                  B, L, 1ull << 32, st, s);
  // Transition k: h = fp16(LN(z0 + t_1 + .. + t_{k-1})), t_k = fp16(ffn(h))
  for (int k = 1; k <= w->n_transitions && r == TMU_OK; ++k) {
    const tmu_cond_transition_weights* tw = &w->transitions[k - 1];
    terms.n = k;
    r = wide ? launch_lnr<256, kRowTerms16>(nullptr, nullptr, 0, 0, &terms, tw->ln_w, tw->ln_b, h, cells, s)
             : launch_lnr<128, kRowTerms16>(nullptr, nullptr, 0, 0, &terms, tw->ln_w, tw->ln_b, h, cells, s);
    if (r) break;
    __half* tk = const_cast<__half*>(terms.src[k]);
    r = wide ? launch_k4_h<256>(h, tk, tw, B, L, hidden, 1ull << 34, st, s)
             : launch_k4_h<128>(h, tk, tw, B, L, hidden, 1ull << 35, st, s);
  }
  if (r) return r;
  // Stage D: h = fp16(LN(z)) without affine, bias = fp16(fp16(h @ bias_w^T) + bias_b), transposed store
  terms.n = w->n_transitions + 1;
  r = wide ? launch_lnr<256, kRowTerms16>(nullptr, nullptr, 0, 0, &terms, nullptr, nullptr, h, cells, s)
           : launch_lnr<128, kRowTerms16>(nullptr, nullptr, 0, 0, &terms, nullptr, nullptr, h, cells, s);
  if (r) return r;
  return launch_k6g<k6::kEpiBiasT>(h, c_pair, w->bias_w, c_pair, n_bias, plain_sched(c_pair), out, w->bias_b, heads,
                                   nullptr, nullptr, B, L, 1ull << 36, st, s);
}

size_t tmu_parcae_workspace_bytes(int B, int L, int c_z) {
  if (B < 1 || L < 1 || c_z < 1) return 0;
  return static_cast<size_t>(B) * L * L * 3 * c_z * 2;
}

int tmu_parcae_step(const float* z, const float* z_init, const float* refined, const tmu_parcae_weights* w,
                    float* z_out, int B, int L, int c_z, void* workspace, size_t workspace_bytes, void* status,
                    void* stream) {
  if (B < 1 || L < 1) return fail(TMU_ERR_INVALID_ARGUMENT, "B and L must be positive");
  if (L > 8192 || B > 65535) return fail(TMU_ERR_UNSUPPORTED, "L > 8192");
  if (c_z != 128 && c_z != 256) return fail(TMU_ERR_UNSUPPORTED, "c_z must be 128 or 256");
  if (w == nullptr || !w->ln_w || !w->ln_b || !w->a || !w->b_split)
    return fail(TMU_ERR_INVALID_ARGUMENT, "parcae weights missing");
  if (!z || !z_init || !refined || !z_out || !workspace || !status) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL tensor");
  if (workspace_bytes < tmu_parcae_workspace_bytes(B, L, c_z))
    return fail(TMU_ERR_WORKSPACE_TOO_SMALL, "workspace too small");
  const void* al[] = {z, z_init, refined, z_out, workspace, w->ln_w, w->ln_b, w->a, w->b_split};
  for (const void* q : al)
    if (!aligned16(q)) return fail(TMU_ERR_MISALIGNED, "pointer not 16-byte aligned");
  DeviceStatus* st = static_cast<DeviceStatus*>(status);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long cells = static_cast<long long>(B) * L * L;
  // LN(z_init + refined), split into three bf16 parts [x0 | x1 | x2]
  int r = c_z == 256 ? launch_lnr<256, kRowSum32, lnr::kOutBf16x3>(z_init, refined, c_z, c_z, nullptr, w->ln_w, w->ln_b,
                                                                  workspace, cells, s)
                     : launch_lnr<128, kRowSum32, lnr::kOutBf16x3>(z_init, refined, c_z, c_z, nullptr, w->ln_w, w->ln_b,
                                                                  workspace, cells, s);
  if (r) return r;
  // the six products x_i B_j with i + j <= 2, smallest first, each over the c_z / 64 K atoms
  static const int pairs[6][2] = {{2, 0}, {1, 1}, {0, 2}, {1, 0}, {0, 1}, {0, 0}};
  K6Sched sc;
  sc.nsteps = 0;
  for (const auto& pr : pairs)
    for (int k = 0; k < c_z / 64; ++k) {
      sc.a_coord[sc.nsteps] = static_cast<short>(pr[0] * c_z + 64 * k);
      sc.w_coord[sc.nsteps] = static_cast<short>(pr[1] * c_z + 64 * k);
      ++sc.nsteps;
    }
  return launch_k6g<k6::kEpiAxpy, true>(workspace, 3 * c_z, w->b_split, 3 * c_z, c_z, sc, z_out, nullptr, 0, z,
                                        w->a, B, L, 1ull << 38, st, s);
}

int tmu_ipc_export(const void* ptr, void* handle, unsigned long long* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL argument");
  CUdeviceptr base = 0;
  int st = allocation_base(ptr, &base);
  if (st) return st;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == TMU_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<CUdeviceptr>(ptr) - base;
  return TMU_OK;
}

int tmu_ipc_import(const void* handle, unsigned long long offset, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *ptr = static_cast<uint8_t*>(base) + offset;
  return TMU_OK;
}

int tmu_ipc_close(void* ptr) {
  if (ptr == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL argument");
  CUdeviceptr base = 0;
  int st = allocation_base(ptr, &base);
  if (st) return st;
  cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void*>(base));
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int tmu_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (dst == nullptr || src == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL argument");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "cudaMemcpyAsync");
}

int tmu_copy2d_async(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width, size_t height,
                     void* stream) {
  if (dst == nullptr || src == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "NULL argument");
  if (width > dst_pitch || width > src_pitch) return fail(TMU_ERR_INVALID_ARGUMENT, "width exceeds a pitch");
  cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width, height, cudaMemcpyDeviceToDevice,
                                    static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "cudaMemcpy2DAsync");
}

int tmu_selftest_wait_timeout(void* status, unsigned long long timeout_ns, void* stream) {
  if (status == nullptr) return fail(TMU_ERR_INVALID_ARGUMENT, "status is NULL");
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<DeviceStatus*>(status),
                                                                       timeout_ns);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TMU_OK : cuda_fail(e, "launch wait_timeout_kernel");
}

}  // extern "C"
