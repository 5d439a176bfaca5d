/*
 * convrot_b200.h -- C ABI of libconvrot_b200.so, the sm_100a (B200) ConvRot
 * W4A4 linear.
 *
 * Every entry point takes device pointers, element counts and a cudaStream_t
 * (passed as void*, NULL = legacy default stream), enqueues its kernels on
 * that stream and returns at once.  No entry point allocates device memory:
 * the caller owns every buffer.  The library itself holds two device arrays
 * per device it is loaded on, for as long as the process lives: a 4-byte
 * error word, and the fixed CONVROT_LINEAR_STATIC_SCRATCH_BYTES (64 MiB)
 * intermediate of convrot_w4a4_linear_static.  Return value: CONVROT_OK (0)
 * or a negative status; convrot_last_error() then gives a message
 * (thread-local).
 *
 * Each function names the reference interface it replaces, as
 * path:line in Lumenbeing/convrot-mlx (src/convrot_mlx/core.py).
 *
 * Conventions shared by all entry points
 *   - matrices are row-major and densely packed (leading dimension = columns);
 *   - "dtype" codes: CONVROT_F32, CONVROT_F16, CONVROT_BF16;
 *   - int4 packing: two's-complement nibbles, element 2j in the low nibble
 *     and 2j+1 in the high nibble of byte j (core.py:97-120);
 *   - weight layouts: CONVROT_LAYOUT_NK = (N, K/2) bytes, packed along K
 *     ("packed-nk-low-nibble-even-feature", core.py:1253-1254);
 *     CONVROT_LAYOUT_KN = (K, N/2) bytes, packed along N
 *     ("packed-kn-low-nibble-even-output", core.py:1248-1250).
 */
#ifndef CONVROT_B200_H
#define CONVROT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define CONVROT_OK 0
#define CONVROT_ERR_INVALID (-1)     /* bad shape, pointer, alignment or argument */
#define CONVROT_ERR_UNSUPPORTED (-2) /* valid for the reference, not for this build */
#define CONVROT_ERR_CUDA (-3)        /* a CUDA runtime / driver call failed */

/* dtype codes */
#define CONVROT_F32 0
#define CONVROT_F16 1
#define CONVROT_BF16 2

/* weight layouts */
#define CONVROT_LAYOUT_NK 0
#define CONVROT_LAYOUT_KN 1

/* ABI version of this header (major * 100 + minor). */
#define CONVROT_ABI_VERSION 100
int convrot_abi_version(void);

/* Message for the last non-zero status returned on this thread. */
const char* convrot_last_error(void);

/*
 * Fused rotate + row quantize, int8 codes.
 * Replaces metal_fused_prepare_convrot_activation_i8 (core.py:456-484; Metal
 * kernel core.py:307-327).  x: (rows, features) of `dtype`; q_i8: (rows,
 * features) int8 codes in [-7, 7]; scales: (rows,) float32 row scales.
 * group_size in {16, 64, 256, 1024} (the reference fuses 64 and 256 and
 * rotates any power of four eagerly, core.py:50-94); features % group_size == 0.
 * group_size 1 skips the rotation (quantize_signed_int4_rowwise,
 * core.py:149-158; then features % 32 == 0).
 */
int convrot_prepare_i8(const void* x, int dtype, int64_t rows, int64_t features,
                       int group_size, int8_t* q_i8, float* scales, void* stream);

/*
 * Fused rotate + row quantize, packed int4 codes.
 * Replaces metal_fused_prepare_convrot_activation (core.py:425-453; Metal
 * kernel core.py:205-304), prepare_convrot_activation (core.py:161-167),
 * compiled_prepare_convrot_activation (core.py:174) and, applied to a dense
 * (out, in) weight, quantize_convrot_weight (core.py:514-527).
 * q_packed: (rows, features / 2) bytes.
 */
int convrot_prepare_packed(const void* x, int dtype, int64_t rows, int64_t features,
                           int group_size, uint8_t* q_packed, float* scales, void* stream);

/*
 * Normalized regular-Hadamard rotation only, output in the input dtype.
 * Replaces metal_fused_rotate_convrot_activation (core.py:487-511; Metal
 * kernel core.py:330-370) and regular_hadamard (core.py:64-94).
 */
int convrot_rotate(const void* x, int dtype, int64_t rows, int64_t features,
                   int group_size, void* out, void* stream);

/*
 * Modulated LayerNorm fused into the prep: the int8 codes and row scales of
 * convrot_prepare_i8 applied to xm = bf16(fma(bf16(LayerNorm(x)),
 * bf16(1 + scale), shift)), the input of a FLUX-style DiT projection, with x
 * read once.  LayerNorm has no affine terms: mean and variance of the row in
 * float32, y = bf16((x - mean) * rsqrt(var + eps)).  shift / scale: one
 * bfloat16 vector of `features` per sample, sample s at s * mod_stride
 * elements (mod_stride % 8 == 0); row r belongs to sample r / rows_per_mod.
 * x bfloat16 only; group_size 64 or 256.  Bit for bit convrot_prepare_i8 of
 * the same xm; against a separate layer_norm + addcmul only the float32 order
 * of the row statistics differs, which can move a code by one.
 * No reference counterpart: it fuses the activation-preparation pass into the
 * producing op, the cost the reference names in docs/design.md:54-64 (its
 * prep alone is core.py:456-484).
 */
int convrot_modnorm_prepare_i8(const void* x, int dtype, int64_t rows, int64_t features, int group_size,
                               const void* shift, const void* scale, int64_t rows_per_mod, int64_t mod_stride,
                               float eps, int8_t* q_i8, float* scales, void* stream);

/*
 * The prep of a FLUX single block's output-projection input fused into its
 * producer: the int8 codes and row scales of convrot_prepare_i8 applied to
 * row r = [a[r, 0:da], gelu_tanh(m[r, 0:dm])] -- the attention output and
 * the MLP half of the block's input projection -- read straight from the two
 * tensors (row strides a_stride and m_stride elements, multiples of 8;
 * da % 16 == 0).  gelu_tanh(x) = 0.5 x (1 + tanh(0.7978845608028654 (x +
 * 0.044715 x^3))) in float32 with each product and sum rounded separately,
 * then one bf16 rounding.  bfloat16 only; group_size 64 or 256.  Bit for bit
 * convrot_prepare_i8 of the concatenated row.  No reference counterpart: the
 * same fusion of the preparation pass into the producing op as
 * convrot_modnorm_prepare_i8.
 */
int convrot_gelu_concat_prepare_i8(const void* a, int64_t a_stride, int64_t da, const void* m, int64_t m_stride,
                                   int64_t dm, int64_t rows, int group_size, int8_t* q_i8, float* scales,
                                   void* stream);

/*
 * Packed int4 -> int8.  Replaces metal_unpack_signed_int4 (core.py:1014-1027;
 * Metal kernel core.py:915-922) and unpack_signed_int4 (core.py:108-120).
 * packed: n_bytes bytes; out: 2 * n_bytes int8 values in [-8, 7].
 */
int convrot_unpack_int4(const uint8_t* packed, int64_t n_bytes, int8_t* out, void* stream);

/*
 * int8 -> packed int4 (values are taken modulo 16).  Replaces
 * pack_signed_int4 (core.py:97-105).  n_values must be even.
 */
int convrot_pack_int4(const int8_t* values, int64_t n_values, uint8_t* out, void* stream);

/*
 * Transpose a packed (rows, 2 * packed_cols) int4 matrix into a packed
 * (2 * packed_cols, rows) one: NK -> KN (repack_nk_weight_for_mpp,
 * core.py:123-133) and KN -> NK (repack_mpp_weight_to_nk, core.py:136-146).
 * rows must be even.  out: (2 * packed_cols, rows / 2) bytes.
 */
int convrot_repack_int4_transpose(const uint8_t* in, int64_t rows, int64_t packed_cols,
                                  uint8_t* out, void* stream);

/*
 * W4A4 linear: out[m, n] = T(float(sum_k a[m,k] w[n,k]) * xscales[m] *
 * wscales[n] + bias[n]) with an exact int32 dot (tcgen05 kind::i8) and the
 * epilogue fused.  Replaces mpp_w4a4_int8_matmul (core.py:1088-1120; Metal
 * K6 core.py:839-874 + epilogue K9 core.py:925-937), and, with layout NK,
 * the math of packed_w4a4_matmul* (core.py:745-828), expanded_fp32 /
 * reference_w4a4_matmul (core.py:1155-1207).
 * act: (m, k) int8 codes; qweight: packed `layout`; xscales (m,), wscales
 * (n,), bias (n,) float32 (bias may be NULL = zeros); out: (m, n) of
 * out_dtype.  k % 32 == 0; layout KN needs n even.
 */
int convrot_w4a4_gemm(const int8_t* act, const uint8_t* qweight, int layout,
                      const float* xscales, const float* wscales, const float* bias,
                      void* out, int out_dtype, int64_t m, int64_t n, int64_t k,
                      void* stream);

/*
 * W4A16 linear: out[m, n] = T(fl(dots[m, n] * wscales[n]) + bias[n]) with
 * dots = sum_k act[m, k] * w[k, n] accumulated in float32 (tcgen05
 * kind::f16; the nibbles are expanded to exact 16-bit integers in shared
 * memory).  Replaces mpp_w4a16_matmul (core.py:1123-1152; Metal K7
 * core.py:877-912, launched at core.py:961-969).  act: (m, k) rotated activations of act_dtype (bfloat16
 * or float16); qweight: packed `layout` (the reference passes K x packed-N);
 * wscales / bias (n,) float32 (bias may be NULL); out: (m, n) of out_dtype.
 * k % 64 == 0; layout KN needs n % 32 == 0 (16-byte weight rows for TMA).
 * The summation order differs from the reference's float32 matmul: results
 * agree to float32 rounding, not bit for bit.
 */
int convrot_w4a16_gemm(const void* act, int act_dtype, const uint8_t* qweight, int layout,
                       const float* wscales, const float* bias, void* out, int out_dtype,
                       int64_t m, int64_t n, int64_t k, void* stream);

/*
 * Tensor-parallel W4A4 (column split of N across the GPUs of one node): the
 * GEMM of this rank's shard -- qweight / wscales / bias hold columns
 * [col_offset, col_offset + n) of the full layer -- whose epilogue writes
 * every output tile into each of the n_outs (1..8) destinations at
 * dst[i * ldc + col_offset + j]: this GPU's full (m, ldc) output and the
 * peers' (device pointers valid on this GPU, e.g. symmetric memory), so the
 * all-gather of the outputs over NVLink overlaps the GEMM tile by tile.
 * Follow it with convrot_peer_barrier before any rank reads its full output.
 * No reference counterpart: the reference runs on one Apple GPU; this is the
 * multi-GPU form of mpp_w4a4_int8_matmul (core.py:1088-1120).  Needs
 * k % 128 == 0 and, for KN, n % 32 == 0.  outs: host array of n_outs device
 * pointers.
 */
int convrot_w4a4_gemm_gather(const int8_t* act, const uint8_t* qweight, int layout,
                             const float* xscales, const float* wscales, const float* bias,
                             void* const* outs, int n_outs, int64_t ldc, int64_t col_offset,
                             int out_dtype, int64_t m, int64_t n, int64_t k, void* stream);

/*
 * Flag barrier across `world` (1..8) GPUs of one node.  flag_arrays: host
 * array of `world` device pointers, valid on this GPU, to each rank's
 * (world,) uint32 flag array (zero-initialised, mapped by every rank).
 * Writes `epoch` (> 0, increasing per call) into slot `rank` of every array
 * with system-scope release stores, then waits, bounded by 2 s, until this
 * rank's array holds `epoch` in every slot (device error code 31 on time-out,
 * see convrot_take_device_error).  No reference counterpart.
 */
int convrot_peer_barrier(uint32_t* const* flag_arrays, int world, int rank, uint32_t epoch,
                         void* stream);

/*
 * A strided block copy on a copy engine (cudaMemcpy2DAsync, device to
 * device): rows x width_bytes, pitches in bytes.  dst may be a peer GPU's
 * memory mapped into this one (symmetric memory).  The tensor-parallel layer
 * pushes each M-chunk of its column shard into every rank's output with it,
 * overlapping the next chunk's GEMM; follow the copies with
 * convrot_peer_barrier.  No reference counterpart.
 */
int convrot_copy_2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t width_bytes,
                    int64_t rows, void* stream);

/*
 * The W4A4 linear in one call that allocates nothing: convrot_prepare_i8
 * followed by convrot_w4a4_gemm, with the int8 codes and row scales between
 * them kept in a fixed device array inside the library instead of a buffer
 * from the caller.  It is for callers that cannot allocate device memory: a
 * plugin that its host engine hands only input and output buffers, or code
 * whose host framework reserves the device's memory for its own allocator.
 * No counterpart in the reference (there the framework allocates).
 *   - The array holds CONVROT_LINEAR_STATIC_SCRATCH_BYTES: the codes of
 *     m x k (rounded up to 256 bytes) plus 4 * m bytes of scales must fit
 *     (m x k up to about 67 million), else CONVROT_ERR_UNSUPPORTED.  Every
 *     GPU that loads the library holds the array until the process exits.
 *   - The first call on a device looks up the array's device address on
 *     that device; made while `stream` is capturing, it is refused with
 *     CONVROT_ERR_UNSUPPORTED (make one call outside capture first).
 *   - Every argument check of convrot_w4a4_gemm runs before anything is
 *     enqueued: a rejected call touches neither the GPU nor the array.
 *   - All calls share the one array: calls whose work overlaps on the GPU
 *     (different streams, or other host threads) race and must not overlap.
 *     Every call rewrites all of the array it reads, so nothing from an
 *     earlier call carries over.
 * Arguments as convrot_prepare_i8 (x, x_dtype, group_size) and
 * convrot_w4a4_gemm (qweight ... stream).
 */
#define CONVROT_LINEAR_STATIC_SCRATCH_BYTES (64LL << 20)
int convrot_w4a4_linear_static(const void* x, int x_dtype, int group_size,
                               const uint8_t* qweight, int layout, const float* wscales,
                               const float* bias, void* out, int out_dtype, int64_t m, int64_t n,
                               int64_t k, void* stream);

/*
 * Diagnostics: which kernel convrot_w4a4_gemm runs.  route 0 (the default):
 * the register-fragment GEMV kernel for m <= 8 (K x packed-N with n % 16 ==
 * 0, or N x packed-K), else the swap-AB kernel for m <= 8 (k % 128 == 0;
 * K x packed-N with n % 32 == 0), else the CTA-pair kernel where it applies
 * (k % 128 == 0; K x packed-N with n % 32 == 0), else the one-CTA kernel;
 * route 1: the one-CTA kernel
 * for every shape; route 2: the CTA-pair kernel wherever it applies (never
 * a small-m one); route 3: the swap-AB kernel wherever it applies (m <=
 * 64); route 4: the register-fragment GEMV kernel wherever it applies
 * (m <= 8; K x packed-N with n % 16 == 0, or N x packed-K).  All give the
 * same bits.  Process-wide; for tests and A/B timing.  No reference
 * counterpart.
 */
int convrot_set_gemm_route(int route);

/*
 * Diagnostics: every wait inside the tcgen05 kernels is bounded; a kernel
 * whose wait times out stops early and records a non-zero code in a
 * device-side word.  This reads and clears that word (0 = no time-out).  It
 * synchronizes the current device.  No reference counterpart (the reference
 * has no failure detection beyond shape checks).  Codes (the first recorded
 * wins): 1-7 one-CTA W4A4 GEMM; 11-19 CTA-pair GEMM (11/12 copy slot free
 * for A / packed weights, 13 accumulator buffer free, 14 A stage landed,
 * 15 expanded weights ready, 16 final MMA drain, 17 packed weights landed,
 * 18 expanded-weight slot free, 19 accumulator ready); 31 peer flag barrier;
 * 41 staged prep row copy; 51-57 swap-AB small-m GEMM (51 packed-weight
 * slot free, 52 activation stage landed, 53 expanded weights ready, 54
 * packed weights landed, 55 expanded-weight slot free, 56 final MMA drain,
 * 57 activation slot free).
 */
int convrot_take_device_error(int* code);

#ifdef __cplusplus
}
#endif

#endif /* CONVROT_B200_H */
