/*
 * bitsparse.h -- C ABI of the B200 (sm_100a) BitSparse activation-compression
 * library (libbitsparse_b200.so).
 *
 * The format is the reference's tile-wise bitmask format (Maxzhu123/bitsparse,
 * lib_sparse/src/triton_kernels.py:1-17): a dense row-major [M, N] matrix is
 * cut into 64x64 tiles in grid-row-major order; each tile has a 512-byte
 * bitmask (bit j of byte b <=> tile element 8b+j, row-major in the tile, set
 * iff the element is > 0); `prefix` is uint32[T+1] with prefix[0] = 0 and
 * prefix[t+1] = prefix[t] + popcount(tile t); `vals` holds the positive
 * elements in (tile, row, column) order starting at logical index
 * `vals_offset`, either raw (bf16 / fp8 bytes) or as a continuous 15-bit
 * (bf16) / 7-bit (fp8) sign-dropped bitstream (lib_sparse/src/bitpacking.py).
 *
 * Conventions of every entry point:
 *  - all pointers are DEVICE pointers on the current CUDA device, except
 *    where stated; nothing is allocated and nothing is freed;
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default);
 *    all work is stream ordered and asynchronous, there is no host sync;
 *  - the return value is BS_OK or a BS_ERR_* code for argument errors
 *    found on the host; errors found on the device (capacity overflow, a
 *    bounded wait that gave up) are OR-ed into the optional `status` word
 *    (device int32*), which the caller reads when it chooses to.
 * Each declaration names the reference interface it replaces (file:line in
 * Maxzhu123/bitsparse).
 */
#ifndef BITSPARSE_B200_H
#define BITSPARSE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
enum {
  BS_OK = 0,
  BS_ERR_SHAPE = 1,     /* negative / too large sizes, bad batch slice      */
  BS_ERR_DTYPE = 2,     /* unsupported dtype or dtype combination           */
  BS_ERR_ALIGN = 3,     /* a pointer that must be aligned is not            */
  BS_ERR_CAPACITY = 4,  /* host-detectable capacity problem                 */
  BS_ERR_LAUNCH = 5,    /* a CUDA launch failed (cudaGetLastError)          */
  BS_ERR_ARG = 6,       /* NULL where a pointer is required, bad flag       */
  BS_ERR_WORKSPACE = 7, /* workspace too small                              */
  BS_ERR_TOO_LARGE = 8  /* beyond a fixed maximum (bs_compress_noalloc)     */
};

/* Device status bits (OR-ed into *status by kernels). */
enum {
  BS_STATUS_CAPACITY = 1, /* vals storage too small: writes were clipped    */
  BS_STATUS_TIMEOUT = 2   /* a bounded device-side wait gave up (results invalid) */
};

/* Element types.  Codes 1/2 equal the reference's pack codecs
 * (lib_sparse/bitsparse.py:8-18). */
enum {
  BS_BF16 = 0,
  BS_E4M3 = 1, /* float8_e4m3fn */
  BS_E5M2 = 2, /* float8_e5m2   */
  BS_F32 = 3
};

/* FP8 quantiser semantics, OR-ed into the dtype argument of bs_fp8_scale,
 * bs_quantize_e4m3 and (with quant_scale) bs_compress, and passed as the
 * fp8_flags argument of the fused FFN entry points.  0 (default): eager
 * PyTorch's to_fp8 arithmetic (bf16 input: scale = bf16(amax / 448), q =
 * e4m3(bf16(x / scale))), which the CPU golden fixtures of the reference
 * hold.  BS_FP8_COMPILED: the arithmetic of the reference's
 * @torch.compile'd to_fp8 on a GPU (lib_sparse/fp8.py:123-129): scale =
 * amax * (1/448) in fp32, q = e4m3(x / scale) with the fp32
 * division of Triton's `/` (PTX div.full.f32) and no intermediate rounding. */
#define BS_FP8_COMPILED 0x100

/* Tile geometry (lib_sparse/config.py:5-6, lib_sparse/bitsparse.py:120-127). */
#define BS_BLOCK_M 64
#define BS_BLOCK_N 64
#define BS_TILE_NUMEL 4096
#define BS_TILE_BYTES 512

/* Library version string, e.g. "bitsparse_b200 0.1 sm_100a". Host pointer. */
const char *bs_version(void);

/* Bytes of workspace bs_compress needs for `num_tiles` tiles (per-partition
 * counts and running totals, about 2 bytes per tile).  Zero the workspace
 * once before its first use (and again after a launch that reported
 * BS_STATUS_TIMEOUT); the library keeps it consistent between launches, so
 * no clearing is queued per call -- the counts of each launch carry an epoch
 * kept in the workspace, which also makes the calls safe to capture in a
 * CUDA graph.  Launches that may overlap on the GPU (different streams) must
 * use different workspaces. */
size_t bs_compress_workspace_bytes(int64_t num_tiles);

/* Fused compress: dense [M, N] (row stride `ld` elements) -> bitmask
 * uint8[T*512], prefix uint32[T+1] and the compacted values in one pass
 * over the input: a persistent kernel (TMA-fed, values compacted in shared
 * memory, bases from per-partition counts published by the other CTAs,
 * waits bounded) when the input base is 16-byte aligned, the row stride is a
 * multiple of 16 bytes and raw `vals` is 16-byte aligned; otherwise (and for
 * BS_F32 input) a count kernel followed by a compact kernel that re-reads
 * the input in reverse order so its most recently counted part comes from
 * L2.
 *
 * Replaces the whole of dense_to_tilesparse (lib_sparse/src/functions.py:55-99):
 * tile_pack (lib_sparse/src/triton_operators.py:21-33), the torch.cumsum
 * prefix (lib_sparse/src/functions.py:33-40), compact_vals
 * (lib_sparse/src/triton_operators.py:36-115, raw and pack_sbit paths) and
 * the TensorBuffer offset update (lib_sparse/src/functions.py:73-92).
 *
 *  in_dtype     BS_BF16, BS_E4M3, BS_E5M2 (stored as-is) or, with
 *               `quant_scale` != NULL, BS_BF16 / BS_F32 quantised in the
 *               kernel to e4m3fn as to_fp8 does (lib_sparse/fp8.py:123-129):
 *               q = e4m3(x / scale) (bf16 input: x / scale rounded to bf16
 *               first); the bitmask is taken from q (q > 0).
 *  quant_scale  device float* (fp32 scale) or NULL.
 *  quant_out    with quant_scale: optional device uint8* [M, N] (row stride
 *               N) receiving the dense e4m3 tensor, or NULL.
 *  vals         raw: element storage (bf16 or 1-byte fp8); pack_sbit:
 *               byte stream addressed as 32-bit words (4-byte aligned).
 *  vals_capacity  raw: elements; pack_sbit: bytes.
 *  arena_offset NULL for standalone storage (values start at 0; in
 *               pack_sbit mode the bytes after the payload up to
 *               vals_capacity are zeroed) or a device int64* holding the
 *               TensorBuffer's running offset: values start at
 *               off = *arena_offset (rounded up to a multiple of 8 when
 *               pack_sbit) and *arena_offset becomes off + nnz.
 *  vals_offset_out optional device int64*: receives `off`.
 *  nnz_out      optional device int64*: receives the total nonzero count.
 */
int bs_compress(const void *dense, int in_dtype, int64_t M, int64_t N,
                int64_t ld, const float *quant_scale, uint8_t *quant_out,
                uint8_t *bitmask, uint32_t *prefix, void *vals,
                int64_t vals_capacity, int pack_sbit, int64_t *arena_offset,
                int64_t *vals_offset_out, int64_t *nnz_out, void *workspace,
                size_t workspace_bytes, int32_t *status, void *stream);

/* Fused bias + ReLU + compress for bf16 input z [M, N]: h = relu(bf16(z +
 * bias)) (the fp32 sum rounded once to bf16, as torch adds bf16 tensors;
 * strictly negative values become +0, -0 and NaN pass through, as
 * torch.relu), h written densely to relu_out [M, N] (row stride relu_ld)
 * and compressed exactly as bs_compress compresses it -- one read of z.
 * The forward of FFNRelu (lib_sparse/layers.py:84-94: z = x W1^T + b1,
 * relu, compress) in one pass.  Needs the one-pass path (z, bias, relu_out
 * and raw vals 16-byte aligned, row strides multiples of 16 bytes);
 * returns BS_ERR_ALIGN otherwise, and the caller falls back to separate
 * steps.  Other arguments as bs_compress. */
int bs_compress_bias_relu(const void *z, int64_t M, int64_t N, int64_t ld,
                          const void *bias, void *relu_out, int64_t relu_ld,
                          uint8_t *bitmask, uint32_t *prefix, void *vals,
                          int64_t vals_capacity, int pack_sbit, int64_t *arena_offset,
                          int64_t *vals_offset_out, int64_t *nnz_out, void *workspace,
                          size_t workspace_bytes, int32_t *status, void *stream);

/* FP8 form of bs_compress_bias_relu: h = relu(bf16(z + bias)) quantised to
 * e4m3 with *scale_h (to_fp8's quantiser, lib_sparse/fp8.py:127) and
 * compressed; side_out (optional, e4m3 [M, N], row stride N) receives the
 * quantised h, or with scale_side != NULL the quantised squared activation
 * e4m3(bf16(h * h) / *scale_side) (Relu2Linear's GEMM input,
 * lib_sparse/layers.py:118-123).  The scales come from
 * bs_fp8_scales_bias_relu.  BS_ERR_ALIGN when the one-pass kernel cannot
 * read z. */
int bs_compress_bias_relu_fp8(const void *z, int64_t M, int64_t N, int64_t ld,
                              const void *bias, const float *scale_h,
                              const float *scale_side, uint8_t *side_out,
                              uint8_t *bitmask, uint32_t *prefix, void *vals,
                              int64_t vals_capacity, int pack_sbit, int64_t *arena_offset,
                              int64_t *vals_offset_out, int64_t *nnz_out, void *workspace,
                              size_t workspace_bytes, int fp8_flags, int32_t *status,
                              void *stream);

/* to_fp8 scales for the fused FFN forward without materialising h =
 * relu(bf16(z + bias)): *scale_h = max(bf16(amax(h) / 448), 1e-9) and,
 * with scale_h2 != NULL, the same rule for h2 = bf16(h * h), whose amax is
 * bf16(amax(h)^2) (rounding is monotonic and h >= 0).  One pass over z;
 * amax_ws as in bs_fp8_scale. */
int bs_fp8_scales_bias_relu(const void *z, int64_t M, int64_t N, int64_t ld,
                            const void *bias, uint32_t *amax_ws, float *scale_h,
                            float *scale_h2, int fp8_flags, void *stream);

/* bs_compress without any device allocation, for callers that cannot call
 * cudaMalloc (code running inside an allocator or a hook where allocating is
 * forbidden, hosts without a device allocator).  No counterpart in the
 * reference.  Same arguments and results as bs_compress minus the workspace:
 * the scan scratch is a fixed 2 MiB + 128 B device array inside the library
 * (held on every GPU that loads it until the process exits), so the tensor
 * may have at most bs_compress_noalloc_max_tiles() 64x64 tiles (262144, e.g.
 * 16384 x 65536 elements); larger tensors return BS_ERR_TOO_LARGE.  The
 * first call on a device looks up the array's device address (make that
 * first call before any stream capture; the address is not looked up again,
 * so do not use this entry point on a device after cudaDeviceReset).  Every
 * argument is checked before anything is queued; a call that passes clears
 * the scratch it uses with cudaMemsetAsync on `stream`.  All calls share the
 * array, so calls that overlap on the GPU race -- serialise them. */
int bs_compress_noalloc(const void *dense, int in_dtype, int64_t M, int64_t N,
                        int64_t ld, const float *quant_scale, uint8_t *quant_out,
                        uint8_t *bitmask, uint32_t *prefix, void *vals,
                        int64_t vals_capacity, int pack_sbit, int64_t *arena_offset,
                        int64_t *vals_offset_out, int64_t *nnz_out, int32_t *status,
                        void *stream);

/* Largest tile count bs_compress_noalloc accepts. */
size_t bs_compress_noalloc_max_tiles(void);

/* Per-tile bitmask and nonzero counts only (no values): the reference's
 * tile_pack (lib_sparse/src/triton_operators.py:21-33,
 * lib_sparse/src/triton_kernels.py:63-97).  counts is int32[T]. */
int bs_tile_pack(const void *dense, int dtype, int64_t M, int64_t N,
                 int64_t ld, int32_t *counts, uint8_t *bitmask, void *stream);

/* Reconstruct a batch of tiles into a dense [batch_rows, K] slice.
 * Replaces unpack_batch_ (lib_sparse/src/triton_operators.py:118-138) and,
 * with relu2 = 1, unpack_relu2_batch_ (:141-162).
 *
 *  store_dtype  BS_BF16 / BS_E4M3 / BS_E5M2 (the BitsparseTensor dtype).
 *  out          relu2 = 0: elements of store_dtype; relu2 = 1: bf16.
 *  out_ld       row stride of `out` in elements.
 *  vals_offset  device int64* (the BitsparseTensor's vals_offset).
 *  scale        relu2 = 1 only: optional device float*; the output is then
 *               multiplied by scale^2 exactly as the reference's separate
 *               `output.mul_(scale.square())` does (fused here).
 *  Tile pid of the batch is tile (first_m_tile + pid / grid_n) * grid_n +
 *  pid % grid_n; its elements go to rows (pid / grid_n) * 64 + r < batch_rows
 *  and columns (pid % grid_n) * 64 + c < K of `out`.
 */
int bs_unpack(const void *vals, const uint8_t *bitmask, const uint32_t *prefix,
              const int64_t *vals_offset, int store_dtype, int pack_sbit,
              void *out, int64_t out_ld, int64_t first_m_tile, int64_t grid_n,
              int64_t K, int64_t batch_rows, int64_t num_tiles_in_batch,
              int relu2, const float *scale, void *stream);

/* to_fp8's quantiser e4m3(bf16(x / *scale)) (lib_sparse/fp8.py:127) on a
 * bf16 [R, C] tensor x (row stride ld), written to q [R, C] (row stride
 * ldq) and/or qT [C, R] (row stride ldqT, the transposed copy) -- the
 * reference's to_fp8 followed by the column-major copy its FP8 GEMM makes
 * of an operand (lib_sparse/fp8.py:15-17), in one read of x.  Either
 * output may be NULL. */
int bs_quantize_e4m3_2d(const void *x, int64_t R, int64_t C, int64_t ld, const float *scale,
                        uint8_t *q, int64_t ldq, uint8_t *qT, int64_t ldqT, int fp8_flags,
                        void *stream);

/* Whether the quantisers may take the plain estimate x * (1 / *scale) for
 * every bf16 x at this scale (fp8_flags: BS_FP8_COMPILED or 0): *out = 1 if
 * an exhaustive check over the bf16 codes that can reach an e4m3 rounding
 * boundary finds the estimate's code equal to the definition's for each,
 * else 0.  The compress and quantise kernels run the same check per CTA and
 * divide where it answers 0; this entry point reports the answer (tests,
 * diagnostics).  out: one device int. */
int bs_fp8_estimate_exact(const float *scale, int fp8_flags, int *out, void *stream);

/* Status of the reconstruct kernels of the current device (bs_unpack has
 * no status argument): *status_out = BS_STATUS_* bits OR-ed since the last
 * reset (BS_STATUS_TIMEOUT: a bounded wait on the bulk copies of the
 * persistent reconstruct gave up).  Synchronous; reset != 0 clears it. */
int bs_unpack_status(int32_t *status_out, int reset);

/* In place grad <- bit ? grad : 0 for a bf16 [M, N] gradient (row stride
 * ld).  Replaces mask_with_bitmask_ (lib_sparse/src/triton_operators.py:165-175,
 * lib_sparse/src/triton_kernels.py:249-276). */
int bs_mask_with_bitmask(void *grad, int grad_dtype, int64_t M, int64_t N,
                         int64_t ld, const uint8_t *bitmask, void *stream);

/* The B operand of the fp8 dW GEMM of Relu2Linear (AspRelu2B,
 * lib_sparse/src/sparse_matmul.py:91-132 with the FP8 matmul of
 * lib_sparse/fp8.py:52-115) straight from the compressed fp8 tensor [M, N]:
 * the ReLU^2 reconstruction of bs_unpack (relu2 = 1) quantised by to_fp8 --
 * its scale, written to *qscale_out, is derived from the largest stored code
 * (the reconstruction is non-decreasing in the stored value) -- and written
 * transposed into outT [N, M] (row stride out_ld >= M), i.e. the [M, N]
 * operand in column-major order.  Raw storage only (not pack_sbit).
 * code_ws: one device uint32 of scratch, zero before the call (left zero). */
int bs_unpack_relu2_fp8t(const void *vals, const uint8_t *bitmask, const uint32_t *prefix,
                         const int64_t *vals_offset, int store_dtype, int64_t M, int64_t N,
                         const float *scale, float k, uint32_t *code_ws, float *qscale_out,
                         void *outT, int64_t out_ld, int fp8_flags, void *stream);

/* In place grad <- bit ? grad * (2 * k * r) : 0, r gathered from the stored
 * values, then (scale != NULL) grad *= scale.  Replaces relu2_grad_sparse_
 * (lib_sparse/src/triton_operators.py:178-202,
 * lib_sparse/src/triton_kernels.py:288-330). */
int bs_relu2_grad(void *grad, int grad_dtype, int64_t M, int64_t N, int64_t ld,
                  const void *vals, const uint8_t *bitmask,
                  const uint32_t *prefix, const int64_t *vals_offset,
                  int store_dtype, int pack_sbit, const float *scale,
                  void *stream);

/* C[M, N] = A[M, K] @ B[K, N] on the tcgen05 tensor cores (bf16 operands,
 * fp32 accumulation, bf16 result rounded to nearest even), with the ReLU
 * mask fused into the epilogue when `mask` != NULL: `mask` is the bitmask of
 * a bitsparse [M, N] tensor and every element whose bit is clear is written
 * as +0.  With the bitmask of the saved activation h this is the backward of
 * ReluLinear, grad_z = (grad_y @ W2) masked by h > 0 (lib_sparse/layers.py:38-51
 * followed by mask_with_bitmask_, lib_sparse/src/triton_kernels.py:249-276),
 * without the dense grad_h reaching memory.  A, B, C row-major with row
 * strides lda >= K, ldb >= N, ldc >= N elements; A and B 16-byte aligned
 * with strides that are multiples of 8 elements (BS_ERR_ALIGN otherwise). */
int bs_gemm_bf16_mask(const void *A, int64_t lda, const void *B, int64_t ldb,
                      void *C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                      const uint8_t *mask, int32_t *status, void *stream);

/* The backward of Relu2Linear for bf16 storage in one tcgen05 GEMM:
 * C = (A @ B) with the ReLU^2 gradient applied in the epilogue --
 * C[i, j] = bit ? bf16(float(bf16(acc)) * (2 k r)) : +0, r the stored value
 * of the bitsparse [M, N] tensor h = relu(z) at (i, j) (raw bf16 storage:
 * `vals` 16-byte aligned, its `bitmask`, `prefix`, device `vals_offset`),
 * k = RELU2_SCALE.  Replaces grad_h = matmul(grad_output, W) followed by
 * relu2_grad_sparse_ (lib_sparse/layers.py:146-147,
 * lib_sparse/src/triton_kernels.py:288-330) with the same roundings,
 * without the dense grad_h reaching memory.  Operands as bs_gemm_bf16_mask. */
int bs_gemm_bf16_relu2(const void *A, int64_t lda, const void *B, int64_t ldb,
                       void *C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                       const void *vals, const uint8_t *bitmask, const uint32_t *prefix,
                       const int64_t *vals_offset, float k, int32_t *status, void *stream);

/* C[M, N] = bf16((A @ Bt^T) * (*scale_a) * (*scale_b)) for e4m3 operands on
 * the tcgen05 tensor cores (kind::f8f6f4, fp32 accumulation): the FP8 GEMM
 * with tensor-wise scales that MatmulFp8 issues through F.scaled_mm
 * (lib_sparse/fp8.py:25-49, 52-115).  A [M, K] and Bt [N, K] (B column-major,
 * as scaled_mm takes it) with unit column stride, row strides lda, ldb >= K
 * bytes, multiples of 16, bases 16-byte aligned (BS_ERR_ALIGN otherwise);
 * C bf16 row-major, row stride ldc >= N; scales device fp32 scalars. */
int bs_gemm_fp8(const void *A, int64_t lda, const void *Bt, int64_t ldb, void *C,
                int64_t ldc, int64_t M, int64_t N, int64_t K, const float *scale_a,
                const float *scale_b, int32_t *status, void *stream);

/* bs_gemm_fp8 with the ReLU^2 gradient of an e4m3-stored activation in the
 * epilogue: g = bf16(acc * sa * sb) (the FP8 GEMM's output), then
 * C[i, j] = bit ? bf16(float(bf16(g * 2 k r)) * (*hscale)) : +0, r the stored
 * e4m3 value of the bitsparse [M, N] tensor (raw storage: `vals` 16-byte
 * aligned, `bitmask`, `prefix`, device `vals_offset`) and hscale its
 * per-tensor scale (NULL: no scaling).  The backward of Relu2Linear in FP8
 * (lib_sparse/layers.py:146-147: grad_h = matmul(grad_output, W, fp8) then
 * relu2_grad_sparse_, lib_sparse/src/triton_kernels.py:288-330 and the
 * grad.mul_(scale) of lib_sparse/src/triton_operators.py:200-201) in one
 * kernel.  Operands as bs_gemm_fp8. */
int bs_gemm_fp8_relu2(const void *A, int64_t lda, const void *Bt, int64_t ldb, void *C,
                      int64_t ldc, int64_t M, int64_t N, int64_t K, const float *scale_a,
                      const float *scale_b, const void *vals, const uint8_t *bitmask,
                      const uint32_t *prefix, const int64_t *vals_offset, float k,
                      const float *hscale, int32_t *status, void *stream);

/* The weight gradient of the FFN's second linear with the reconstruct fused
 * into the GEMM (AspB / AspRelu2B, lib_sparse/src/sparse_matmul.py:9-47 and
 * :91-132, called from lib_sparse/layers.py:58 and :142):
 *   C[D, H] = g^T . h        (relu2 = 0)
 *   C[D, H] = g^T . (k h^2)  (relu2 = 1; k must be 1, the reference's RELU2_SCALE)
 * g: bf16 [T, D] row-major (row stride ldg elements, 16-byte aligned base
 * and row stride); h: the bf16 bitsparse tensor [T, H] (vals 16-byte
 * aligned, bitmask, prefix, vals_offset as bs_compress wrote them, raw
 * storage, 64 x 64 tiles); C: bf16 [D, H] (row stride ldc).  Each 64 x 64
 * tile of h is expanded from its compressed form straight into the tensor
 * cores' shared-memory operand; the dense h is never written.  fp32
 * accumulation (over K splits: fp32 partials summed in order), C rounded to
 * bf16 once.  workspace: bs_gemm_unpack_dw_workspace_bytes(T, D, H) bytes,
 * 16-byte aligned (may be null when that is 0; BS_ERR_WORKSPACE when short).
 * status: as bs_compress (bounded waits).  BS_ERR_ALIGN when g, vals or
 * bitmask cannot be read by TMA / bulk copies. */
int bs_gemm_unpack_dw(const void *g, int64_t ldg, int64_t T, int64_t D, const void *vals,
                      const uint8_t *bitmask, const uint32_t *prefix,
                      const int64_t *vals_offset, int64_t H, int relu2, float k, void *C,
                      int64_t ldc, void *workspace, size_t workspace_bytes, int32_t *status,
                      void *stream);

/* Bytes of workspace bs_gemm_unpack_dw needs for these sizes on the current
 * device: when the output has too few tiles to occupy every SM pair, K is
 * split and the fp32 partials (splits x D x H) live there; 0 otherwise. */
size_t bs_gemm_unpack_dw_workspace_bytes(int64_t T, int64_t D, int64_t H);

/* Per-tile FP8 scale mode -- an extension: the reference's to_fp8 uses one
 * scale per tensor (lib_sparse/fp8.py:123-129).  A bf16 [M, N] tensor (row
 * stride ld; TMA-readable: 16-byte aligned base and row stride, else
 * BS_ERR_ALIGN) is quantised to e4m3 with one scale per 64 x 64 tile and
 * compressed in one pass: for tile t, amax_t = max |x| over its elements
 * (NaN ignored), tile_scales[t] = amax_t / 448 and each code is
 * e4m3(x * (448 / amax_t)) -- the quotients and the product correctly
 * rounded in fp32, the cast rounding to nearest even (an all-zero tile: scale
 * 1, codes 0).  The positive codes are then stored exactly as bs_compress
 * stores e4m3 values (bitmask, prefix, values, arena offset, pack_sbit).
 * tile_scales: float[num_tiles].  Other arguments as bs_compress. */
int bs_compress_fp8_tile_scaled(const void *dense, int64_t M, int64_t N, int64_t ld,
                                float *tile_scales, uint8_t *bitmask, uint32_t *prefix,
                                void *vals, int64_t vals_capacity, int pack_sbit,
                                int64_t *arena_offset, int64_t *vals_offset_out,
                                int64_t *nnz_out, void *workspace, size_t workspace_bytes,
                                int32_t *status, void *stream);

/* Reconstruct of a per-tile-scaled e4m3 tensor into bf16: out =
 * bf16(value(code) * tile_scales[t]) (fp32 product, round to nearest even),
 * 0 where the bitmask bit is clear.  Batch arguments as bs_unpack. */
int bs_unpack_tile_scaled(const void *vals, const uint8_t *bitmask, const uint32_t *prefix,
                          const int64_t *vals_offset, int pack_sbit, const float *tile_scales,
                          void *out, int64_t out_ld, int64_t first_m_tile, int64_t grid_n,
                          int64_t K, int64_t batch_rows, int64_t num_tiles_in_batch,
                          void *stream);

/* Per-tensor fp8 scale of to_fp8 (lib_sparse/fp8.py:123-129):
 * *scale_out = max(amax(|x|) / 448, 1e-9), with the amax / 448 rounded to
 * bf16 for bf16 input (eager PyTorch semantics).  `amax_ws` is a device
 * uint32 the caller zero-fills before the call (one word of scratch). */
int bs_fp8_scale(const void *x, int dtype, int64_t numel, uint32_t *amax_ws,
                 float *scale_out, void *stream);

/* q = e4m3fn(x / *scale) elementwise over `numel` elements of a bf16 or
 * fp32 tensor -- the quantise step of to_fp8 (lib_sparse/fp8.py:127).
 * Eager semantics round a bf16 input's quotient to bf16 first; with
 * BS_FP8_COMPILED in dtype the quotient is Triton's fp32 division, as the
 * reference's compiled to_fp8 computes it.  Quotients beyond +-464 (never
 * produced by to_fp8's own scales, |x / scale| <= 448 * (1 + 2^-8))
 * saturate to +-448 for bf16 input, as Triton's cast does.  The kernel
 * quantises by the estimate x * (1 / scale) where bs_fp8_estimate_exact
 * holds at the scale and divides otherwise: same codes.  x 16-byte aligned,
 * q 8-byte aligned. */
int bs_quantize_e4m3(const void *x, int dtype, int64_t numel, const float *scale,
                     uint8_t *q, void *stream);

/* dst[c][r] = src[r][c] for 1-byte elements (fp8): the operand transposes
 * that the reference's FP8 GEMM wrapper makes with .T.contiguous()
 * (lib_sparse/fp8.py:39-43, :107-110) because cuBLASLt's FP8 GEMM takes A
 * row-major and B column-major.  src [rows, cols] row stride ld_src, dst
 * [cols, rows] row stride ld_dst. */
int bs_transpose_b8(const void *src, int64_t rows, int64_t cols, int64_t ld_src,
                    void *dst, int64_t ld_dst, void *stream);

/* Values only, with tile offsets from an existing prefix: the reference's
 * compact_vals (lib_sparse/src/triton_operators.py:36-115,
 * lib_sparse/src/triton_kernels.py:105-146, lib_sparse/src/bitpacking.py:58-117).
 * The bitmask is recomputed from `dense` (it is a function of it).
 * vals_offset: device int64* logical start of the values (NULL = 0).
 * vals_capacity: elements (raw) or bytes (pack_sbit). */
int bs_compact_vals(const void *dense, int dtype, int64_t M, int64_t N, int64_t ld,
                    const uint32_t *prefix, void *vals, int64_t vals_capacity,
                    int pack_sbit, const int64_t *vals_offset, int32_t *status,
                    void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BITSPARSE_B200_H */
