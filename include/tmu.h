/*
 * tmu.h -- C ABI of the B200 (sm_100a) triangle multiplicative update.
 *
 * This is the drop-in boundary for the hot path of abhi0raj/esmfold2-mlx's folding trunk
 * (paths below are relative to the reference's src/esmfold2_mlx/).  The reference runs the
 * tri-mul as MLX ops plus three Metal kernels compiled through mx.fast.metal_kernel; each entry
 * point here replaces one or more of those calls:
 *
 *   tmu_project_gate   <- proj = n @ w_in; gate_cf(proj, mask, c)        mlx_trunk_kernels.py:214-216, :85-97
 *                         (and the input LayerNorm: mlx_trunk_kernels.py:233 / mlx_trunk.py:81)
 *   tmu_contract       <- a @ b.swapaxes(2,3) | a.swapaxes(2,3) @ b       mlx_trunk_kernels.py:219, mlx_trunk.py:84-88
 *   tmu_emit_residual  <- ln_cf_to_cl; @ w_emit; n @ w_out_gate; resgate  mlx_trunk_kernels.py:221-227, :152-160, :195-203
 *   tmu_trimul         <- one whole triangle update z + _trimul(z)        mlx_trunk_kernels.py:210-229, mlx_trunk.py:79-90,94-95
 *
 * Conventions
 *   - All tensors are device pointers to fp16 (IEEE binary16) unless stated; biases are fp32.
 *   - z, z_out: [B, L, L, c_z] channels-last, contiguous, 16-byte aligned.  z_out may equal z.
 *   - mask: [B, L, L] fp16 pair mask (reference: pair_attention_mask cast to fp16), or NULL for
 *     an all-ones mask (var_mlx_trunk.py:40-43 skips the multiply in that case).
 *   - a, b, x: [B*c, L, Lpad] channel-major, Lpad = tmu_row_pitch(L) (= L rounded up to 8);
 *     the pad columns are never read.
 *   - stream: a cudaStream_t passed as void*; every launch goes on it, nothing synchronises.
 *   - status: device memory of at least TMU_STATUS_BYTES (16-byte aligned) holding the device-side
 *     status word; kernels record a bounded-wait timeout there.  It keeps two records: the
 *     current call's first error (tmu_read_status; cleared by the first kernel of tmu_trimul and
 *     tmu_pair_block) and the first error since the block was last zeroed by tmu_reset_status
 *     (tmu_read_first_error; no kernel clears it, so one read covers a whole sequence of calls).
 *   - Widths: c_z == c, 128 or 256 (the released ESMFold2 trunk's width, mlx_trunk.py:4);
 *     1 <= L <= 8192, B*c <= 65535.  Other sizes return TMU_ERR_UNSUPPORTED.  At c_z = 256,
 *     z_out must not overlap z (two CTAs share each tile's z): TMU_ERR_INVALID_ARGUMENT.
 *   - Return value: TMU_OK or a TMU_ERR_* code (never aborts the process).  Device-side
 *     conditions (TMU_ERR_DEVICE_TIMEOUT, TMU_ERR_SMEM_LAYOUT) land in the status word.
 */
#ifndef TMU_H_
#define TMU_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TMU_OK 0
#define TMU_ERR_INVALID_ARGUMENT 1
#define TMU_ERR_MISALIGNED 2
#define TMU_ERR_WORKSPACE_TOO_SMALL 3
#define TMU_ERR_UNSUPPORTED 4
#define TMU_ERR_CUDA 5
#define TMU_ERR_DEVICE_TIMEOUT 6
#define TMU_ERR_ARCH 7
#define TMU_ERR_DRIVER 8
#define TMU_ERR_SMEM_LAYOUT 9 /* device status: a kernel found its shared memory misaligned and did nothing */

#define TMU_STATUS_BYTES 256

/* Weights of one triangle update, device pointers (mlx_trunk.py:40-55 `_trimul_params`).
 * w_proj rows follow tmu_proj_row_order(); the signal-a rows already carry the fp16 scheme's
 * 1/256 pre-scale (mlx_trunk.py:47-48).  Biases are optional (NULL = the reference's form);
 * b_emit and b_gate must be both set or both NULL. */
typedef struct tmu_trimul_weights {
  const void* ln_in_w;  /* [c_z]       norm_start.weight */
  const void* ln_in_b;  /* [c_z]       norm_start.bias */
  const void* w_proj;   /* [4c, c_z]   proj_bundle.weight rows, packed order */
  const float* b_proj;  /* [4c]        fp32, packed order, or NULL */
  const void* ln_mix_w; /* [c]         norm_mix.weight */
  const void* ln_mix_b; /* [c]         norm_mix.bias */
  const void* w_emit;   /* [c_z, c]    proj_emit.weight */
  const float* b_emit;  /* [c_z]       fp32 or NULL */
  const void* w_gate;   /* [c_z, c_z]  proj_gate.weight */
  const float* b_gate;  /* [c_z]       fp32 or NULL */
} tmu_trimul_weights;

/* Library version string. */
const char* tmu_version(void);

/* Name of a status code ("TMU_OK", "TMU_ERR_UNSUPPORTED", ...). */
const char* tmu_status_name(int status);

/* Last CUDA error string seen by the library on this thread (for TMU_ERR_CUDA / _DRIVER). */
const char* tmu_last_error(void);

/* Checks that the current device is a Blackwell sm_100 part the kernels were built for. */
int tmu_device_check(void);

/* Row pitch (elements) of the channel-major a, b, x buffers for sequence length L. */
int tmu_row_pitch(int L);

/* Packed-row order of proj_bundle.weight: order[r] is the proj_bundle row that becomes packed
 * row r (blocks of c rows: signal a, gate a, signal b, gate b).  `order` must hold 4*c ints. */
int tmu_proj_row_order(int c, int* order);

/* Bytes of workspace tmu_trimul needs: status word + a + b + x. */
size_t tmu_workspace_bytes(int B, int L, int c_z, int c);

/* Default bound for every device-side wait, in nanoseconds (initially 2e9).  Returns the old value. */
unsigned long long tmu_set_wait_timeout_ns(unsigned long long ns);

/* Zero the status word (async on `stream`). */
int tmu_reset_status(void* status, void* stream);

/* Synchronise `stream`, then copy the status word to the host.  *code is TMU_OK or
 * TMU_ERR_DEVICE_TIMEOUT; *site identifies the wait that gave up (0 if none). */
int tmu_read_status(const void* status, void* stream, int* code, int* site);

/* Like tmu_read_status, but returns the first error recorded in `status` since it was last zeroed
 * by tmu_reset_status, whichever call recorded it: a caller that runs many calls on one status
 * word (a 24-block trunk pass) zeroes it once, runs the calls and reads it once. */
int tmu_read_first_error(const void* status, void* stream, int* code, int* site);

/* Launch-span trace, a measurement aid (no counterpart in the reference).  tmu_trace_arm zeroes a
 * status block and switches its trace on (async on `stream`); every kernel launched with that
 * block as its status word then records, in %globaltimer nanoseconds, the earliest time one of its
 * CTAs passed its dependency wait and the latest time one finished.  Giving each launch of a
 * chain its own armed block times the kernels inside a programmatic-dependent-launch chain,
 * which events between the launches would break.  tmu_trace_read synchronises `stream` and
 * returns the two times (t_start = UINT64_MAX if no kernel ran with the block).  Traced: the
 * tri-mul kernels (tmu_project_gate, tmu_contract, tmu_emit_residual and their _ex forms) and
 * tmu_transition. */
int tmu_trace_arm(void* status, void* stream);
int tmu_trace_read(const void* status, void* stream, unsigned long long* t_start, unsigned long long* t_end);

/* K1: n = LN(z); a, b = gated projections of n, channel-major.  outputs a, b: [B*c, L, Lpad]. */
int tmu_project_gate(const void* z, const void* mask, const tmu_trimul_weights* w, int B, int L, int c_z,
                     int c, void* a, void* b, void* status, void* stream);

/* K2: x[d] = a[d] b[d]^T (outgoing != 0) or a[d]^T b[d] (incoming), d in [0, Bc). fp32 accumulate. */
int tmu_contract(const void* a, const void* b, void* x, int Bc, int L, int outgoing, void* status, void* stream);

/* K3: z_out = z + fp16(LN_mix(x) @ w_emit) * sigmoid(fp16(LN(z) @ w_gate)). */
int tmu_emit_residual(const void* x, const void* z, void* z_out, const tmu_trimul_weights* w, int B, int L,
                      int c_z, int c, float mix_eps, void* status, void* stream);

/* ---- Row slabs (one long sequence sharded over devices; no counterpart in the reference, which
 * runs one device).  A slab is a rows x cols block of the pair grid.  These entry points let a
 * caller run the three stages on slabs and do the exchange between them itself (NCCL):
 *   outgoing: project_gate_ex on the local rows -> all-gather b -> contract_ex -> emit_residual_ex
 *   incoming: all-to-all the local rows into local columns (z^T), project_gate_ex on that
 *             transposed view -> all-gather b' -> contract_ex -> emit_residual_ex on the local rows.
 */
typedef struct tmu_pair_layout {
  int B, rows, cols;                       /* B folds of rows x cols positions */
  long long stride_b, stride_row, stride_col;                 /* z element strides (channels contiguous) */
  long long mask_stride_b, mask_stride_row, mask_stride_col;  /* mask element strides (ignored if no mask) */
} tmu_pair_layout;

/* K1 on a strided rows x cols view: a, b are [B*c, rows, tmu_row_pitch(cols)]. */
int tmu_project_gate_ex(const void* z, const void* mask, const tmu_pair_layout* layout, const tmu_trimul_weights* w,
                        int c_z, int c, void* a, void* b, void* status, void* stream);

/* K2 in the outgoing form on slabs: x[d] (M x N) = a[d] (M x K) b[d]^T, a is [Bc, M, pitch(K)],
 * and b is N / b_rows_per_part consecutive blocks [Bc, b_rows_per_part, pitch(K)] (what an
 * all-gather of the ranks' [Bc, rows, pitch(K)] slabs produces).  With more than one block,
 * b_rows_per_part must be a multiple of 128.  x is [Bc, M, ldx] with rows of ldx elements
 * (ldx = 0: tmu_row_pitch(N)); with ldx > N, x may point at a column block of a wider matrix
 * (16-byte aligned), so the blocks of b can be contracted one at a time as they arrive.
 * max_ctas > 0 caps the kernel's persistent grid (one CTA per SM otherwise), leaving SMs free
 * for kernels that must run alongside it, such as the NCCL transfer of the next block. */
int tmu_contract_ex(const void* a, const void* b, void* x, int Bc, int M, int N, int K, int b_rows_per_part,
                    int ldx, int max_ctas, void* status, void* stream);

/* K3 on a contiguous [B, rows, cols, c_z] slab with x [B*c, rows, pitch(cols)]. */
int tmu_emit_residual_ex(const void* x, const void* z, void* z_out, int B, int rows, int cols,
                         const tmu_trimul_weights* w, int c_z, int c, float mix_eps, void* status, void* stream);

/* K1 -> K2 -> K3: z_out = z + tri-mul(z).  `workspace` of tmu_workspace_bytes() bytes, 256-byte
 * aligned; its first TMU_STATUS_BYTES are the status word (zeroed by this call's first kernel).
 * The kernels are launched with programmatic dependent launch, so each one's set-up overlaps
 * the end of the kernel before it. */
int tmu_trimul(const void* z, void* z_out, const void* mask, const tmu_trimul_weights* w, int B, int L, int c_z,
               int c, int outgoing, float mix_eps, void* workspace, size_t workspace_bytes, void* stream);

/* Size cap of tmu_trimul_noalloc: each of its three channel-major buffers (a, b, x) must fit in
 * this many bytes, i.e. B * c * L * tmu_row_pitch(L) * 2 <= 8 MiB: one fold up to L = 178 at
 * c = 128 and up to L = 128 at c = 256. */
#define TMU_NOALLOC_MAX_BUFFER_BYTES (8u << 20)

/* One triangle update, z_out = z + tri-mul(z), like tmu_trimul but without a workspace argument
 * and without allocating anything.  This entry point has no counterpart in the reference.
 *
 * It is meant for callers that are not allowed to allocate device memory at the moment they
 * run the update: for example a host framework that reserves all device memory up front and
 * forbids allocation inside its execute callback, or a caller that cannot accept the implicit
 * device-wide synchronisation that cudaMalloc/cudaFree bring.  Instead of a caller-provided
 * workspace it uses one fixed scratch array built into this library (3 x 8 MiB plus a 256-byte
 * status word, TMU_NOALLOC_MAX_BUFFER_BYTES per buffer), which every GPU that loads the library
 * holds until the process exits.  Sizes beyond the cap return TMU_ERR_UNSUPPORTED with a message
 * (tmu_last_error); use tmu_trimul for them.  The call itself issues no cudaMalloc or cudaFree.
 *
 * - The first call on each device looks up that device's address of the scratch array
 *   (cudaGetSymbolAddress, with the device current) and caches it for the life of the process:
 *   make that first call before any stream capture on the device, and do not keep using this
 *   entry point after cudaDeviceReset (the cached address would point into the destroyed
 *   context).
 * - At c_z = 256, z_out must not overlap z (TMU_ERR_INVALID_ARGUMENT), as for tmu_trimul.
 * - All calls on a device share the one scratch array, which keeps the previous call's
 *   contents.  The call clears the status word it uses; everything else is rewritten before it
 *   is read.  Calls that can overlap on the GPU (different streams without ordering, or several
 *   host threads) race on the scratch and give wrong results: serialise them.
 * - `status`: device memory of TMU_STATUS_BYTES, 16-byte aligned, for the bounded-wait status word
 *   (read it with tmu_read_status), or NULL to use the scratch's own word, which the caller
 *   cannot read.  The call zeroes the whole status block before its first kernel. */
int tmu_trimul_noalloc(const void* z, void* z_out, const void* mask, const tmu_trimul_weights* w, int B, int L,
                       int c_z, int c, int outgoing, float mix_eps, void* status, void* stream);

/* ---- Pair transition (K4), the third op of a PairUpdateBlock: z_out = z + ffn(LN(z)).
 * Replaces the reference's transition (mlx_trunk.py:96-99; fused path mlx_trunk_kernels.py:236-239):
 * h = fp16(LN(z)), x = fp16(h @ w12^T), SwiGLU s = fp16(fp16(x1 * fp16(sigmoid(x1))) * x2) with
 * x1, x2 the two halves of x (TMU_ACT_RELU: s = relu(x), for synthetic configurations), and
 * z_out = fp16(z + s @ w3^T) with one rounding.  z_out may alias z. */
#define TMU_ACT_SWIGLU 0
#define TMU_ACT_RELU 1

typedef struct tmu_transition_weights {
  const void* ln_w;  /* fp16 [c_z]: norm.weight */
  const void* ln_b;  /* fp16 [c_z]: norm.bias */
  const void* w12;   /* fp16 [2*hidden, c_z] (SwiGLU) or [hidden, c_z] (ReLU): ffn.w12.weight */
  const void* w3;    /* fp16 [c_z, hidden]: ffn.w3.weight */
} tmu_transition_weights;

/* c_z = 128 or 256, hidden a multiple of 64 in [64, 4096]; z [B, L, L, c_z] fp16. */
int tmu_transition(const void* z, void* z_out, const tmu_transition_weights* w, int B, int L, int c_z, int hidden,
                   int activation, void* status, void* stream);

/* ---- One PairUpdateBlock in one call: tri-mul outgoing, tri-mul incoming, then the pair
 * transition, on fp16 z [B, L, L, c_z] (the reference's block_forward, mlx_trunk_kernels.py:232-239;
 * unfused order mlx_trunk.py:93-99).  Seven launches on `stream`, chained with programmatic
 * dependent launch: K1 K2 K3 outgoing, K1 K2 K3 incoming, K4.  z_out may equal z.  At c_z = 128
 * both updates run in place on z_out; at c_z = 256 (whose kernels cannot write over their input)
 * the outgoing update goes to a pair buffer at the end of the workspace.  The workspace
 * (tmu_pair_block_workspace_bytes bytes, 256-byte aligned) starts with the status word, zeroed by
 * the first kernel and shared by all seven (tmu_read_status).  Constraints: those of tmu_trimul
 * and tmu_transition. */
size_t tmu_pair_block_workspace_bytes(int B, int L, int c_z, int c);
int tmu_pair_block(const void* z, void* z_out, const void* mask, const tmu_trimul_weights* w_out,
                   const tmu_trimul_weights* w_in, const tmu_transition_weights* w_tr, int B, int L, int c_z, int c,
                   int hidden, int activation, float mix_eps, void* workspace, size_t workspace_bytes, void* stream);

/* ---- Distogram expected distance (K5), the convergence signal of adaptive recycling
 * (var_adaptive_loops.py:43-46): out[b,i,j] = sum_k softmax((z[b,i,j] + z[b,j,i]) @ w^T + bias)_k
 * * centres[k].  z [B, L, L, c_z] fp16 (c_z = 128 or 256), w fp16 [n_bins, c_z] (the head's
 * weight rounded to fp16), bias fp32 [n_bins] or NULL, centres fp32 [n_bins], out fp32
 * [B, L, L]; n_bins = 128. */
int tmu_disto_expected(const void* z, const void* w, const float* bias, const float* centres, float* out, int B,
                       int L, int c_z, int n_bins, void* status, void* stream);

/* ---- Diffusion pair conditioning (K6 + K4 row mode): the per-fold pair biases of the diffusion
 * head's token transformer.  Replaces pair_biases (mlx_diffusion16.py:81-87 in the pair16
 * precision of the adopted var_mlx_diffusion16 stack; fp32 form mlx_diffusion.py:252-259):
 *   z    = fp16(fp16(LN(concat(z_trunk, rel_pos))) @ proj^T)                  (fp32 from here on)
 *   z   += fp32(fp16(fp16(silu(x1) * x2) @ w3^T)), x = fp16(fp16(LN(z)) @ w12^T)   per transition
 *   bias = fp16(fp16(fp16(LN(z)) @ bias_w^T) + bias_b)       (LN without affine)
 * and out[k, b, h, i, j] = bias[b, i, j, k * heads + h]  ([n_bias / heads, B, heads, L, L]).
 * z_trunk, rel_pos fp32 [B, L, L, c_trunk] and [B, L, L, c_rel]; LayerNorm parameters fp32, matrices fp16 in nn.Linear layout
 * ([out, in]); bias_w [n_bias, c_pair] folds each token block's pair_norm affine into its
 * pair_bias_proj (mlx_diffusion.py:85-89), bias_b fp16 [n_bias]. */
typedef struct tmu_cond_transition_weights {
  const float* ln_w;  /* fp32 [c_pair]: norm.weight */
  const float* ln_b;  /* fp32 [c_pair]: norm.bias */
  const void* w12;    /* fp16 [2*hidden, c_pair]: a_proj.weight rows, then b_proj.weight rows */
  const void* w3;     /* fp16 [c_pair, hidden]: out_proj.weight */
} tmu_cond_transition_weights;

typedef struct tmu_pair_cond_weights {
  const float* ln_w;  /* fp32 [c_trunk + c_rel]: z_input_norm.weight */
  const float* ln_b;  /* fp32 [c_trunk + c_rel]: z_input_norm.bias */
  const void* proj;   /* fp16 [c_pair, c_trunk + c_rel]: z_proj.weight */
  int n_transitions;
  const tmu_cond_transition_weights* transitions; /* [n_transitions] */
  const void* bias_w; /* fp16 [n_bias, c_pair] */
  const void* bias_b; /* fp16 [n_bias] */
} tmu_pair_cond_weights;

/* Bytes of scratch tmu_pair_cond needs: the fp32 residual stream kept as its fp16 terms (z0 and
 * each transition's output: n_transitions + 1 tensors [B, L, L, c_pair]), then one fp16 buffer
 * [B, L, L, max(c_in, c_pair)] for the LayerNorm output each GEMM kernel reads; every tensor
 * starts on a 256-byte boundary.  c_in = c_trunk + c_rel. */
size_t tmu_pair_cond_workspace_bytes(int B, int L, int c_in, int c_pair, int n_transitions);

/* Shapes: c_trunk == c_rel, c_trunk + c_rel in {256, 512}; c_pair in {128, 256}; at most 3
 * transitions; hidden a multiple of 64 in [64, 4096]; n_bias a multiple of 16 in [16, 256],
 * divisible by heads. */
int tmu_pair_cond(const float* z_trunk, const float* rel_pos, const tmu_pair_cond_weights* w, int B, int L,
                  int c_trunk, int c_rel, int c_pair, int hidden, int n_bias, int heads, void* out,
                  void* workspace, size_t workspace_bytes, void* status, void* stream);

/* ---- Parcae step of the 6B release model's recycling loop (var_6b_mlx_loop.py:67-71, fp32 in
 * the reference):  z_out = a * z + LN(z_init + refined) @ B^T, with refined the lm_encoder
 * trunk's output.  z, z_init, refined, z_out fp32 [B, L, L, c_z] (z_out may alias z); a fp32
 * [c_z] (a scalar a is a constant vector); LayerNorm fp32 (parcae_input_norm, eps 1e-5).
 * The GEMM runs on the tensor cores with fp32 accuracy: B is passed split into three bf16 parts,
 * b_split = [B0 | B1 | B2] bf16 [c_z, 3 c_z] with B = B0 + B1 + B2 exactly (B0 = bf16(B),
 * B1 = bf16(B - B0), B2 = bf16(B - B0 - B1)), LN's output is split the same way in the kernel,
 * and the six products x_i B_j with i + j <= 2 accumulate in fp32. */
typedef struct tmu_parcae_weights {
  const float* ln_w;    /* fp32 [c_z]: parcae_input_norm.weight */
  const float* ln_b;    /* fp32 [c_z]: parcae_input_norm.bias */
  const float* a;       /* fp32 [c_z] */
  const void* b_split;  /* bf16 [c_z, 3 c_z] */
} tmu_parcae_weights;

/* Scratch for the split LayerNorm output: bf16 [B, L, L, 3 c_z]. */
size_t tmu_parcae_workspace_bytes(int B, int L, int c_z);

/* c_z = 128 or 256. */
int tmu_parcae_step(const float* z, const float* z_init, const float* refined, const tmu_parcae_weights* w,
                    float* z_out, int B, int L, int c_z, void* workspace, size_t workspace_bytes, void* status,
                    void* stream);

/* ---- Copy-engine exchange for the row-sharded path (no counterpart in the reference).  A rank
 * exports a device buffer with tmu_ipc_export (CUDA IPC handle of the allocation that contains
 * `ptr`, plus ptr's byte offset inside it); a peer process imports it with tmu_ipc_import and
 * copies from it with tmu_copy_async, a cudaMemcpyAsync that the copy engines carry over NVLink,
 * so the transfer uses no SM and no kernel ever reads another GPU's memory.  tmu_ipc_close
 * releases an imported mapping (pass the pointer tmu_ipc_import returned). */
#define TMU_IPC_HANDLE_BYTES 64

int tmu_ipc_export(const void* ptr, void* handle, unsigned long long* offset);
int tmu_ipc_import(const void* handle, unsigned long long offset, void** ptr);
int tmu_ipc_close(void* ptr);
int tmu_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/* A pitched copy by the copy engines (cudaMemcpy2DAsync): `height` rows of `width` bytes from
 * `src` (rows `src_pitch` bytes apart) to `dst` (rows `dst_pitch` bytes apart).  The row-sharded
 * incoming update pulls each peer's block of z rows x this rank's columns with one such copy,
 * which is the all-to-all and its transpose in one transfer; the channel partition pulls each
 * peer's rows of this rank's channels of a and b (and this rank's rows of the peer's channels
 * of x) the same way, one run of rows x pitch elements per channel. */
int tmu_copy2d_async(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width, size_t height,
                     void* stream);

/* Self-test of the bounded-wait machinery: launches one CTA that waits on an mbarrier nothing
 * ever arrives at, with a limit of `timeout_ns`; the kernel must give up, record
 * TMU_ERR_DEVICE_TIMEOUT in `status` and exit.  Returns the launch status. */
int tmu_selftest_wait_timeout(void* status, unsigned long long timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TMU_H_ */
