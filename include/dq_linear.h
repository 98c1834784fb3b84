/*
 * dq_linear.h -- C ABI of the B200 (sm_100a) quantized weight-only linear
 * engine for diffuseR's NF4 and fp8-e4m3 linears.
 *
 * Every entry point takes plain device pointers and sizes plus a CUDA stream,
 * allocates nothing (scratch comes from the caller's workspace), never aborts
 * and returns a dq_status.  Work is enqueued on `stream`; kernels that hit a
 * bounded wait record DQ_ERR_TIMEOUT in a per-device error word readable with
 * dq_device_error().
 *
 * Layouts are the reference's (diffuseR 0.2.2):
 *   x       bf16 [M, K] row-major (any leading dims flattened into M)
 *   packed  uint8 [N*K/2]   NF4 codes, element 2j in the HIGH nibble of byte j
 *   absmax  f32  [N*K/64]   one scale per 64 consecutive weight elements
 *   w8      e4m3fn [N, K]   fp8 weight, per-tensor fp32 scale
 *   bias    bf16 [N] or NULL
 *   y       bf16 [M, N]
 * Requirements: K % 64 == 0 for NF4 (blocks lie inside a weight row),
 * K % 16 == 0 for fp8; x, packed/w8 and y 16-byte aligned.
 */
#ifndef DQ_LINEAR_H
#define DQ_LINEAR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque stream handle: a cudaStream_t (0 = legacy default stream). */
typedef void* dq_stream_t;

typedef enum dq_status {
  DQ_OK = 0,
  DQ_ERR_SHAPE = 1,     /* non-positive size, bad K (see above), length % 64 != 0 */
  DQ_ERR_ALIGN = 2,     /* an operand is not 16-byte aligned */
  DQ_ERR_ARCH = 3,      /* current device is not sm_100 (B200 / GB200) */
  DQ_ERR_LAUNCH = 4,    /* a kernel launch failed */
  DQ_ERR_TIMEOUT = 5,   /* a kernel's bounded wait expired (dq_device_error) */
  DQ_ERR_WORKSPACE = 6, /* workspace NULL or smaller than dq_workspace_size() */
  DQ_ERR_ARG = 7,       /* NULL operand pointer or unknown enum value */
  DQ_ERR_CUDA = 8,      /* another CUDA runtime error */
  DQ_ERR_SCRATCH_LIMIT = 9 /* dq_linear_nf4_noalloc: shape needs more scratch than it has */
} dq_status;

typedef enum dq_format { DQ_FMT_NF4 = 0, DQ_FMT_FP8 = 1 } dq_format;

typedef enum dq_dtype { DQ_DTYPE_F32 = 0, DQ_DTYPE_BF16 = 1 } dq_dtype;

/* Library version string and the ABI revision of this header. */
const char* dq_version(void);
int dq_abi_version(void);
const char* dq_status_string(int status);

/* ---------------------------------------------------------------- quantize
 * NF4 quantizer.  Replaces ltx23_nf4_quantize (R/nf4_ltx23.R:35-61):
 * per 64-element block absmax (f32, clamped >= 1e-12), normalized = w/absmax,
 * code = bucketize(normalized, f32 level midpoints, right = FALSE), two codes
 * per byte (first in the high nibble).  n_elems % 64 == 0.
 * w is f32 or bf16 (w_dtype); outputs packed [n/2] and absmax [n/64]. */
int dq_quantize_nf4(const void* w, int w_dtype, int64_t n_elems,
                    uint8_t* packed, float* absmax, dq_stream_t stream);

/* Per-tensor fp8-e4m3 quantizer.  Replaces the cast branch of flux_quantize
 * (R/quantize_flux.R:406-409) and ltx23_quantize_fp8 (R/fp8_ltx23.R:178-181):
 * scale = max(max|w|, 1e-12) / 448 (f32), w8 = e4m3fn(w / scale).
 * Writes the scale to the device float *scale_out. */
int dq_quantize_fp8(const void* w, int w_dtype, int64_t n_elems,
                    uint8_t* w8, float* scale_out, dq_stream_t stream);

/* -------------------------------------------------------------- dequantize
 * NF4 -> bf16.  Replaces ltx23_nf4_dequantize(dtype = bf16)
 * (R/nf4_ltx23.R:77-115 with the byte LUT of R/jit_ltx23.R:270-281):
 * out = RNE_bf16(bf16(level) * bf16(absmax)), bit-exact. */
int dq_dequant_nf4(const uint8_t* packed, const float* absmax, int64_t n_elems,
                   void* out_bf16, dq_stream_t stream);

/* e4m3 -> bf16.  Replaces the upcast + rescale of ltx23_fp8_linear$forward
 * (R/fp8_ltx23.R:79-80): out = RNE_bf16(e4m3 * bf16(scale)), bit-exact. */
int dq_dequant_fp8(const uint8_t* w8, float scale, int64_t n_elems,
                   void* out_bf16, dq_stream_t stream);

/* ------------------------------------------------------------------ linear
 * Bytes of caller-provided scratch the linear needs for this shape: split-K
 * partial sums for small token counts; for the two-phase plan of large ones
 * the bf16 weight (N*K*2, rounded up to 256) followed by the weight groups'
 * ready counters (4 * (N/256 + 2) bytes, rounded up to 256); else 0.  The
 * contents need no initialization; calls that may run concurrently (on
 * different streams) need distinct workspaces. */
size_t dq_workspace_size(int64_t M, int64_t N, int64_t K, int fmt);

/* y = x . dequant(W)^T + bias, dequantization fused into a tcgen05 GEMM.
 * Replaces ltx23_nf4_linear$forward (R/nf4_ltx23.R:235-246) and the
 * TorchScript nf4_lin (R/jit_ltx23.R:40-50). */
int dq_linear_nf4(const void* x, int64_t M, int64_t K,
                  const uint8_t* packed, const float* absmax,
                  const void* bias, int64_t N, void* y,
                  void* workspace, size_t workspace_bytes, dq_stream_t stream);

/* Same for fp8-e4m3 with a per-tensor scale passed by value.
 * Replaces ltx23_fp8_linear$forward (R/fp8_ltx23.R:70-83). */
int dq_linear_fp8(const void* x, int64_t M, int64_t K,
                  const uint8_t* w8, float scale,
                  const void* bias, int64_t N, void* y,
                  void* workspace, size_t workspace_bytes, dq_stream_t stream);

/* Allocation-free NF4 linear, for callers that cannot allocate device
 * memory: embedders whose device memory is owned by a foreign allocator (the
 * R torch package's caching allocator, for instance) and who have no
 * workspace to lend, and code that must not allocate while it runs (a
 * serving loop with a fixed memory budget).  This entry point has no counterpart in the
 * reference.  Same math and arguments as dq_linear_nf4 minus the workspace:
 * split-K partial sums go to a scratch array built into the library
 * (DQ_NOALLOC_SCRATCH_BYTES = 8 MiB, held on every GPU that loads the
 * library until the process exits).  Large token counts run the fused
 * kernels rather than the two-phase plan, and automatic plans split K only as
 * far as their partial sums fit the array; a split count forced with
 * dq_set_tile_override that needs more returns DQ_ERR_SCRATCH_LIMIT without
 * launching anything (after the same argument checks as dq_linear_nf4).  The first call
 * on a device looks up the array's device address (make that first call
 * before any stream capture).  All calls share the one array: calls whose
 * kernels overlap on the GPU (different streams, no ordering) race on it.
 * Every partial sum is written before it is read, so nothing needs clearing. */
#define DQ_NOALLOC_SCRATCH_BYTES (8u << 20)
int dq_linear_nf4_noalloc(const void* x, int64_t M, int64_t K,
                          const uint8_t* packed, const float* absmax,
                          const void* bias, int64_t N, void* y, dq_stream_t stream);

/* ---------------------------------------------------------------- errors
 * Reads and clears the current device's kernel error word (synchronizes
 * `stream`).  *code receives DQ_OK or DQ_ERR_TIMEOUT. */
int dq_device_error(int* code, dq_stream_t stream);

/* Kernel-configuration override for benchmarking sweeps: x-tile rows
 * (16..256, multiple of 16; 0 = automatic) and split-K count (0 = auto). */
int dq_set_tile_override(int bm, int splits);

/* Kernel-family override for benchmarking: 0 = automatic, 1 = fused, one CTA
 * per tile (128 weight rows), 2 = fused, CTA-pair tiles (256 weight rows,
 * x-tile >= 64), 3 = two-phase: the weight dequantized once into bf16 scratch
 * (part of the workspace) by the bf16 CTA-pair GEMM launch itself, one group
 * of weight tiles ahead of its MMAs (automatic for M >= 1024), 4 = two-phase
 * with the dequantization as a separate launch before the GEMM, 5 = the
 * small-M kernels (weights decoded into warp-MMA registers; M <= 16 and
 * K % 128 == 0, automatic for M <= 8 and for M <= 16 when N >= 32 * SMs):
 * for M <= 8 the weight streamed through a TMA ring in shared memory where
 * K % 256 == 0 (NF4) / K % 128 == 0 (fp8) and the NF4 absmax is 16-byte
 * aligned (automatic for M <= 4), else loaded straight into registers; 6 =
 * the small-M kernel that loads the weight straight into registers, always. */
int dq_set_pair_mode(int mode);

/* ------------------------------------------------- column-parallel linear
 * Tensor parallelism over out_features for one linear (the weight rows split
 * across `world` GPUs of one node, 1 <= world <= 8).  Rank r holds weight rows
 * [r*N/world, (r+1)*N/world): for NF4 the byte range [n0*K/2, n1*K/2) of the
 * reference's packed buffer and [n0*K/64, n1*K/64) of absmax (NF4 blocks are
 * row-local, so a shard needs no repacking), for fp8 those rows of w8 with the
 * shared scalar scale.  Each rank's fused kernel stores its [M, N/world]
 * block straight into EVERY rank's y [M, N] (bf16, columns n0..n1) through
 * peer pointers, then raises its flag in every rank's flag array; the call
 * enqueues a bounded wait (5 s, then DQ_ERR_TIMEOUT in dq_device_error) until
 * this rank's flags show all blocks have landed.  No library collective.
 *
 *   y_ranks[world]    host array of device pointers: rank q's y, mapped here
 *   flag_ranks[world] host array of device pointers: rank q's uint32[world]
 *   counter           this rank's uint32, zero before the first call
 *   epoch             1, 2, 3, ... one per call, the same on every rank
 *
 * Buffers shared between ranks come from dq_tp_buffer_alloc (zero-filled) and
 * are mapped into the other processes with dq_ipc_handle / dq_ipc_open.
 * N % world == 0.  One call in flight per device.  The reference has no
 * multi-GPU path; this is the partitioning of its linear (R/nf4_ltx23.R:235-246,
 * R/fp8_ltx23.R:70-83) over rows of W. */
#define DQ_IPC_HANDLE_BYTES 64
int dq_tp_buffer_alloc(size_t bytes, void** ptr);
int dq_tp_buffer_free(void* ptr);
int dq_ipc_handle(const void* ptr, void* handle_out);
int dq_ipc_open(const void* handle, void** ptr);
int dq_ipc_close(void* ptr);
int dq_tp_linear_nf4(const void* x, int64_t M, int64_t K, const uint8_t* packed_shard,
                     const float* absmax_shard, const void* bias_shard, int64_t N, int rank,
                     int world, void* const* y_ranks, unsigned int* const* flag_ranks,
                     unsigned int* counter, unsigned int epoch, dq_stream_t stream);
int dq_tp_linear_fp8(const void* x, int64_t M, int64_t K, const uint8_t* w8_shard, float scale,
                     const void* bias_shard, int64_t N, int rank, int world, void* const* y_ranks,
                     unsigned int* const* flag_ranks, unsigned int* counter, unsigned int epoch,
                     dq_stream_t stream);

/* The column-parallel linears with a workspace (`dq_workspace_size(M,
 * N / world, K, fmt)` bytes, 16-byte aligned; workspace_bytes must be at least
 * what this rank's shard plan needs): from 1024 tokens each rank then runs the
 * two-phase plan -- its shard's weight decoded once into the workspace by the
 * GEMM launch itself -- whose epilogue stores into every rank's y as above;
 * below that the fused kernels, as without a workspace.  Results are the same
 * bits either way.  NULL workspace: DQ_ERR_WORKSPACE. */
int dq_tp_linear_nf4_ws(const void* x, int64_t M, int64_t K, const uint8_t* packed_shard,
                        const float* absmax_shard, const void* bias_shard, int64_t N, int rank,
                        int world, void* const* y_ranks, unsigned int* const* flag_ranks,
                        unsigned int* counter, unsigned int epoch, void* workspace,
                        size_t workspace_bytes, dq_stream_t stream);
int dq_tp_linear_fp8_ws(const void* x, int64_t M, int64_t K, const uint8_t* w8_shard, float scale,
                        const void* bias_shard, int64_t N, int rank, int world, void* const* y_ranks,
                        unsigned int* const* flag_ranks, unsigned int* counter, unsigned int epoch,
                        void* workspace, size_t workspace_bytes, dq_stream_t stream);

/* The column-parallel linears with a workspace, writing through an NVLink
 * multicast mapping: y_multicast is the multicast address of this call's y
 * buffer (the same offset in every rank's y, as a symmetric-memory multicast
 * object bound to all ranks' y buffers provides), so every 16-byte epilogue
 * store is one `multimem.st` that the NVSwitch replicates into all ranks' y
 * instead of one store per rank.  y_ranks stay required (unicast pointers for
 * stores that are not 16-byte aligned and for nothing else); flags, counter,
 * epoch and the bounded wait are as above.  The same bits as
 * dq_tp_linear_*_ws.  NULL y_multicast: DQ_ERR_ARG. */
int dq_tp_linear_nf4_mc_ws(const void* x, int64_t M, int64_t K, const uint8_t* packed_shard,
                           const float* absmax_shard, const void* bias_shard, int64_t N, int rank,
                           int world, void* const* y_ranks, void* y_multicast,
                           unsigned int* const* flag_ranks, unsigned int* counter,
                           unsigned int epoch, void* workspace, size_t workspace_bytes,
                           dq_stream_t stream);
int dq_tp_linear_fp8_mc_ws(const void* x, int64_t M, int64_t K, const uint8_t* w8_shard,
                           float scale, const void* bias_shard, int64_t N, int rank, int world,
                           void* const* y_ranks, void* y_multicast,
                           unsigned int* const* flag_ranks, unsigned int* counter,
                           unsigned int epoch, void* workspace, size_t workspace_bytes,
                           dq_stream_t stream);

/* The linears with an activation fused into the epilogue: act = DQ_ACT_NONE or
 * DQ_ACT_GELU_TANH, y = bf16(gelu_tanh(bf16(x . W^T + bias))).  Replaces the
 * reference's up-projection followed by nnf_gelu(approximate = "tanh")
 * (ltx23_feed_forward's gelu_proj, R/dit_ltx23_modules.R:500-516, and the
 * FLUX single block's proj_mlp, R/dit_flux_modules.R:311).
 *
 * Gated activations: DQ_ACT_SWIGLU, y = bf16(bf16(silu(g)) * u), replaces the
 * FLUX.2 / Z-Image feed-forward's linear_in followed by silu of its first
 * half times its second half (flux2_feed_forward, R/dit_flux2_modules.R:77-84,
 * and the MLP half of to_qkv_mlp_proj, :148-150); DQ_ACT_GEGLU_TANH, the same
 * with gelu_tanh(g) (a GELU-gated MLP such as Gemma3's).  g and u are the
 * bf16-rounded projections of the gate and up rows.  The weight (and bias)
 * must be in the gated row order: N % 32 == 0 and, for each output feature
 * block b of 16, weight rows 32b .. 32b+15 are the gate rows 16b .. 16b+15
 * and rows 32b+16 .. 32b+31 the up rows of the same features (from the
 * reference's [gate; up] halves: gated row 32b + i = row 16b + i for i < 16,
 * row N/2 + 16b + i - 16 otherwise).  y then has N / 2 columns (ldy >= N / 2);
 * the column-parallel entry points take no gated activation (DQ_ERR_ARG). */
enum { DQ_ACT_NONE = 0, DQ_ACT_GELU_TANH = 1, DQ_ACT_SWIGLU = 2, DQ_ACT_GEGLU_TANH = 3 };
int dq_linear_nf4_ex(const void* x, int64_t M, int64_t K, const uint8_t* packed,
                     const float* absmax, const void* bias, int64_t N, int act, void* y,
                     void* workspace, size_t workspace_bytes, dq_stream_t stream);
int dq_linear_fp8_ex(const void* x, int64_t M, int64_t K, const uint8_t* w8, float scale,
                     const void* bias, int64_t N, int act, void* y, void* workspace,
                     size_t workspace_bytes, dq_stream_t stream);

/* The NF4 / fp8 linear with an activation (as the *_ex entry points) writing
 * y[m * ldy + n] (ldy >= the output width: N, or N / 2 with a gated
 * activation): the output can be a column range of a
 * wider row-major buffer, e.g. one part of a concatenation that the next
 * linear reads whole (no counterpart in the reference, which concatenates
 * tensors with torch_cat).  Everything else as dq_linear_nf4 / dq_linear_fp8. */
int dq_linear_nf4_ld(const void* x, int64_t M, int64_t K, const uint8_t* packed,
                     const float* absmax, const void* bias, int64_t N, int act, void* y,
                     int64_t ldy, void* workspace, size_t workspace_bytes, dq_stream_t stream);
int dq_linear_fp8_ld(const void* x, int64_t M, int64_t K, const uint8_t* w8, float scale,
                     const void* bias, int64_t N, int act, void* y, int64_t ldy, void* workspace,
                     size_t workspace_bytes, dq_stream_t stream);

/* The NF4 linear with the block scales in either dtype: scale_dtype =
 * DQ_DTYPE_F32 (the reference's absmax buffer, f32 [N*K/64]) or DQ_DTYPE_BF16
 * (the same scales repacked at load time as bf16(absmax): the forward casts
 * absmax to bf16 before multiplying (R/nf4_ltx23.R:97, R/jit_ltx23.R:49),
 * so the dequantized weights are bit-identical, with 2 bytes per block
 * instead of 4).  act and ldy as dq_linear_nf4_ld (ldy = 0: the output width).
 * Replaces ltx23_nf4_linear$forward (R/nf4_ltx23.R:235-246). */
int dq_linear_nf4_scaled(const void* x, int64_t M, int64_t K, const uint8_t* packed,
                         const void* absmax, int scale_dtype, const void* bias, int64_t N, int act,
                         void* y, int64_t ldy, void* workspace, size_t workspace_bytes,
                         dq_stream_t stream);

/* NF4 -> bf16 with f32 or bf16 block scales (as dq_linear_nf4_scaled);
 * replaces ltx23_nf4_dequantize (R/nf4_ltx23.R:77-115), bit-exact. */
int dq_dequant_nf4_scaled(const uint8_t* packed, const void* absmax, int scale_dtype,
                          int64_t n_elems, void* out_bf16, dq_stream_t stream);

/* Describes the launch plan dq_linear_* uses for this shape on the current
 * device: *pair = 0 for fused one-CTA tiles (128 weight rows), 1 for fused
 * CTA-pair tiles (256 rows), 2 for the two-phase plan (the bf16 CTA-pair GEMM
 * whose launch also dequantizes the weight into scratch), 3 for the small-M kernel
 * that loads the weight into registers, 4 for the small-M kernel that streams
 * it through a TMA ring (*bm = 8 or 16 tokens; 16, 32 or 64 weight rows per
 * CTA); *bm = x-tile rows, *splits = split-K count, *grid = CTAs launched.  A
 * diagnostic query with no reference counterpart. */
int dq_plan_info(int64_t M, int64_t N, int64_t K, int fmt, int* pair, int* bm, int* splits,
                 int* grid);

#ifdef __cplusplus
}
#endif

#endif /* DQ_LINEAR_H */
