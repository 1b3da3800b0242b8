/*
 * oc_b200.h -- C ABI of the B200 (sm_100a) int4/int2 linear hot path of
 * onecomp_runtime (kizuna-intelligence/onecompression-runtime).
 *
 * Plain C: raw device pointers, sizes, dtype tags and a cudaStream_t. No torch
 * types. Every call is stream-ordered, allocates no device memory and returns an
 * int status (OC_OK == 0); oc_b200_last_error() holds the message of the last
 * failing call on the calling thread.
 *
 * The reference has no native FFI; each entry point below replaces a Python
 * function or a Triton launch of the reference, cited as file:line relative to
 * the reference package root (onecomp_runtime/).
 */
#ifndef OC_B200_H_
#define OC_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* oc_stream_t; /* identical to cudaStream_t */
typedef struct oc_b200_layer oc_b200_layer; /* opaque: host-side metadata of one packed layer */

enum {
  OC_OK = 0,
  OC_ERR_INVALID = 1,     /* bad argument (shape, dtype, alignment, null pointer) */
  OC_ERR_UNSUPPORTED = 2, /* valid request this build does not implement, or not an sm_100 device */
  OC_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
  OC_ERR_DEVICE = 4,      /* a kernel reported a bounded wait that gave up (see oc_b200_read_device_error) */
  OC_ERR_WORKSPACE = 5    /* workspace missing or too small */
};

enum { OC_DT_F16 = 0, OC_DT_BF16 = 1, OC_DT_F32 = 2 };

enum {
  OC_OPT_GEMM_PATH = 1,    /* 0 auto (M<=16 -> split-K GEMV, else tcgen05), 1 force GEMV, 2 force tcgen05 */
  OC_OPT_TC_TILE = 2,      /* tokens per tcgen05 tile: 0 auto, 128, 192, 256, 384, 448 */
  OC_OPT_GEMV_CTAS = 3,    /* GEMV CTAs per SM that split-K sizing fills in one wave (default 2) */
  OC_OPT_GEMV_IMPL = 4,    /* decode kernel for uniform-group layers: 0 tcgen05, 1 TMA + mma.sync split-K,
                              2 cp.async + mma.sync, 3 stream-K TMA + mma.sync with the act-order gather inside
                              (M <= 8 and at least 256 columns; otherwise 1), 4 (default) integer tensor
                              cores: activations prepared as 16-bit fixed point per 128-k stage (two 8-bit
                              digits) with the act-order gather, u8 codes x digits MMAs (4-bit codes, M <= 8;
                              otherwise 1) */
  OC_OPT_TC_PAIR = 5,      /* tcgen05 GEMM on CTA pairs (cta_group::2): 0 auto, 1 single CTAs (default), 2 pairs */
  OC_OPT_WAIT_US = 6,      /* failure tests: bound of the TMA decode GEMV's pipeline waits in microseconds
                              (0, the default: 2 s); drains of copies in flight keep the 2 s bound */
  OC_OPT_TEST_STALL = 7,   /* failure tests: s > 0 makes the first CTA of each TMA decode GEMV leave stage
                              s - 1 unissued, so a wait runs out, the kernel records OC_ERR_DEVICE's code,
                              skips that tile's output and leaves its tickets re-armed; 0 (default) off */
  OC_OPT_TC_MAX_CTAS = 8,  /* persistent tcgen05 GEMMs (GPTQ and row-packed): at most this many CTAs,
                              0 (default) one per SM; a tensor-parallel job leaves SMs to the NCCL
                              all-reduce that overlaps the next chunk's GEMM */
  OC_OPT_GEMV_PREP = 9     /* integer decode GEMV, one token, no act-order permutation: 1 (default) each CTA
                              prepares the activations of its K split itself (at most 20 stages of 128 k per
                              split, else as 0), 0 a separate preparation launch into the workspace (always
                              used for M > 1 and act-order layers); identical results */
};

/* ---- library / device ------------------------------------------------------ */
int oc_b200_abi_version(void);
const char* oc_b200_last_error(void);
/* OC_OK when `device` is an sm_100 (B200-class) GPU. Mirrors the build-time
 * capability gate of backend.resolve_backend (backend.py:103-144). */
int oc_b200_device_check(int device);
int oc_b200_set_option(int key, int value);
/* Current value of an OC_OPT_* option (process-wide). */
int oc_b200_get_option(int key, int* value);
/* Copies the kernels' device error word into *code (0 = none) and clears it.
 * Synchronises `stream`. */
int oc_b200_read_device_error(int* code, oc_stream_t stream);

/* ---- unpack / pack / dequant ---------------------------------------------- */
/* Replaces quant_utils.unpack_int_weights (quant_utils.py:36-42): qweight
 * int32 [K/(32/wbits), N] -> w_int int32 [N, K]. */
int oc_b200_gptq_unpack(const int32_t* qweight, int K, int N, int wbits, int32_t* w_int, oc_stream_t stream);
/* Replaces quant_utils.unpack_zeros (quant_utils.py:45-47): qzeros int32
 * [G, N/(32/wbits)] -> zeros int32 [G, N] (stored values, no v1 restore). */
int oc_b200_gptq_unpack_zeros(const int32_t* qzeros, int G, int N, int wbits, int32_t* zeros, oc_stream_t stream);
/* Replaces _pack_int4_weights (layers/fused_int4_linear.py:76-91), any wbits
 * dividing 32: w_int int32 [N, K] -> qweight int32 [ceil(K/pf), N]. */
int oc_b200_gptq_pack(const int32_t* w_int, int N, int K, int wbits, int32_t* qweight, oc_stream_t stream);
/* Replaces quant_utils.dequant_gptq_to_fp (quant_utils.py:50-69), bit-exact:
 * out[n, k] = RNE_out( f32(s[g,n]) * (q[n,k] - z[g,n]) ), g = g_idx[k] (g_idx may be
 * NULL: g = k / groupsize). v1 != 0 applies the AutoGPTQ-v1 zero restore
 * (z + 1) & mask (quant_utils.py:64-65). out is [N, K] (nn.Linear layout). */
int oc_b200_gptq_dequant(const int32_t* qweight, const int32_t* qzeros, const void* scales, int scales_dtype,
                         const int64_t* g_idx, int K, int N, int G, int groupsize, int wbits, int v1, void* out,
                         int out_dtype, oc_stream_t stream);
/* Replaces quant_utils.dequant_extra_u8_to_weight (quant_utils.py:72-103),
 * bit-exact including its roundings in the output dtype (f16, bf16 or f32).
 * qweight_u8 is [N, ld_bytes] (low nibble = even k); scales/zeros [N, G] f16/bf16/f32. */
int oc_b200_rtn_dequant(const uint8_t* qweight_u8, int64_t ld_bytes, const void* scales, int scales_dtype,
                        const void* zeros, int zeros_dtype, int K, int N, int G, void* out, int out_dtype,
                        oc_stream_t stream);
/* Replaces PackedEmbedding.forward (packed_linear.py:92-104: three row gathers, then
 * dequant_extra_u8_to_weight): out[i, :] = the RTN-dequantized row ids[i] of a packed table
 * qweight_u8 [vocab, ld_bytes] with scales/zeros [vocab, G], bit-exact with the reference.
 * Negative ids count from the end of the table; ids outside [-vocab, vocab) give a zero row
 * and set the device error word (read with oc_b200_read_device_error). out_dtype f16, bf16
 * or f32 (the reference returns the scales' dtype). */
int oc_b200_rtn_embedding(const int64_t* ids, int64_t n_ids, int64_t vocab, const uint8_t* qweight_u8,
                          int64_t ld_bytes, const void* scales, int scales_dtype, const void* zeros, int zeros_dtype,
                          int dim, int G, void* out, int out_dtype, oc_stream_t stream);
/* Replaces layers/dsv4_packed_linear.dequant_dsv4_packed (dsv4_packed_linear.py:22-56),
 * bit-exact. packed is [N, ld_bytes], 8/wbits codes per byte (code j at bits
 * j*wbits). scales/zeros element (n, g) sits at n*stride_n + g*stride_g
 * (covers both the [N, G] and [G, N] layouts); groupsize <= 0: one group per row. */
int oc_b200_dsv4_dequant(const uint8_t* packed, int64_t ld_bytes, int wbits, const void* scales, int scales_dtype,
                         const void* zeros, int zeros_dtype, int64_t stride_n, int64_t stride_g, int groupsize,
                         int K, int N, void* out, int out_dtype, oc_stream_t stream);

/* ---- K re-layout (load time) ----------------------------------------------- */
/* Builds the kernel-side K order used for act-order g_idx and for groupsizes
 * that are not a multiple of 8 (the role of _repack_groups_to_32,
 * fused_int4_linear.py:94-124): qweight_out[w', n] packs, for i < 8, the code of
 * source row k_perm[8w'+i] (or 0 when it is -1). */
int oc_b200_gptq_repack_k(const int32_t* qweight, const int32_t* k_perm, int k_packed, int N, int32_t* qweight_out,
                          oc_stream_t stream);
/* The same for wbits 4 (as above) or 8: an 8-bit qweight_out[w', n] packs, for i < 4, the code of
 * source row k_perm[4w'+i] (k_packed a multiple of 4). The K re-layout of 8-bit act-order layers
 * (PackedGPTQLinear(wbits=8) with g_idx, packed_gptq_linear.py:34-64). */
int oc_b200_gptq_repack_k_ex(const int32_t* qweight, const int32_t* k_perm, int k_packed, int N, int wbits,
                             int32_t* qweight_out, oc_stream_t stream);
/* x_out[m, k'] = x[m, k_perm[k']] (0 when -1); 16-bit elements. */
int oc_b200_permute_cols(const void* x, int64_t ldx, int64_t M, int K, const int32_t* k_perm, int k_packed,
                         void* x_out, oc_stream_t stream);

/* ---- packed GPTQ int4 linear ----------------------------------------------- */
/* Describes one AutoGPTQ int4 layer for the GEMM kernels. Replaces the module
 * state of FusedInt4Linear (fused_int4_linear.py:966-1014),
 * FusedInt4LinearAnyGroup (:646-670), FusedInt4LinearPaddedGroups (:770-811) and
 * PackedGPTQLinear (packed_gptq_linear.py:34-64).
 *   qweight    int32 [k_packed/8, N] in kernel K order
 *   qzeros     int32 [G, N/8], scales [G, N] (f16 or bf16)
 *   k_perm     int32 [k_packed] or NULL: kernel row k' reads activation column
 *              k_perm[k'] (-1 = zero padding); NULL means k_packed == in_features
 *   word_group int32 [k_packed/8] or NULL: group of each 8-row word; NULL means
 *              group = 8*w / groupsize
 * Pointers must stay valid for the handle's lifetime; the handle owns no device memory. */
int oc_b200_gptq_layer_create(const int32_t* qweight, const int32_t* qzeros, const void* scales, int scales_dtype,
                              const int32_t* k_perm, const int32_t* word_group, int in_features, int k_packed,
                              int N, int G, int groupsize, int v1, oc_b200_layer** out);
/* oc_b200_gptq_layer_create with the code width: wbits 4 (as above) or 8. 8-bit layers
 * (quant_utils.py:12-28 with wbits=8; PackedGPTQLinear(wbits=8), packed_gptq_linear.py:66-74)
 * have qweight int32 [in_features/4, N] and qzeros int32 [G, N/4]; oc_b200_gptq_gemm runs
 * them on the decode GEMV (M <= 16) or the tcgen05 GEMM (8-bit stages, exact dequant). They
 * need uniform groups in kernel K order (groupsize 32 or a multiple of 64, no word_group): either
 * k_perm NULL, or an act-order layer whose groups each hold groupsize rows, with k_perm its
 * group-sorted row order (in_features entries, k_packed == in_features) and qweight repacked in
 * that order (oc_b200_gptq_repack_k_ex); N a multiple of 32 and >= 128, in_features >= 64, and
 * 16-byte aligned tensors; other layouts return OC_ERR_UNSUPPORTED. */
int oc_b200_gptq_layer_create_ex(const int32_t* qweight, const int32_t* qzeros, const void* scales, int scales_dtype,
                                 const int32_t* k_perm, const int32_t* word_group, int in_features, int k_packed,
                                 int N, int G, int groupsize, int wbits, int v1, oc_b200_layer** out);
int oc_b200_layer_destroy(oc_b200_layer* layer);
/* Bytes of workspace oc_b200_gptq_gemm needs for M rows. The first
 * 8192 bytes hold split-K tickets that must be zero before the first call on a
 * workspace (every call leaves them zero again). */
size_t oc_b200_gptq_gemm_workspace(const oc_b200_layer* layer, int64_t M);
/* C[M, N] = A[M, in_features] @ dequant(W)^T + bias, fp32 accumulation, bias
 * added in fp32, one rounding to a_dtype (f16/bf16). Replaces fused_int4_gemm /
 * _fused_int4_gemm_kernel (fused_int4_linear.py:388-537, :127-272) and
 * PackedGPTQLinear.forward (packed_gptq_linear.py:66-74). M <= 16 runs the
 * split-K GEMV, larger M the tcgen05 kernel. A rows are lda elements apart
 * (16-byte aligned), C rows ldc apart. */
int oc_b200_gptq_gemm(const oc_b200_layer* layer, const void* a, int a_dtype, int64_t M, int64_t lda,
                      const void* bias, int bias_dtype, void* c, int64_t ldc, void* workspace,
                      size_t workspace_bytes, oc_stream_t stream);
enum { OC_ACT_NONE = 0, OC_ACT_GELU_TANH = 1 };
/* oc_b200_gptq_gemm with a fused epilogue: C = act(A @ W^T + bias) + residual, evaluated in
 * fp32 and rounded once (act: OC_ACT_NONE or OC_ACT_GELU_TANH, torch's approximate="tanh";
 * residual: optional [M, ldr] in a_dtype, may alias C). Folds the activation and residual
 * add that follow the reference's linears in DiT blocks into the GEMM's store. */
int oc_b200_gptq_gemm_ex(const oc_b200_layer* layer, const void* a, int a_dtype, int64_t M, int64_t lda,
                         const void* bias, int bias_dtype, const void* residual, int64_t ldr, int act, void* c,
                         int64_t ldc, void* workspace, size_t workspace_bytes, oc_stream_t stream);
/* No counterpart in the reference. The decode GEMV of oc_b200_gptq_gemm (1 <= M <= 16, same
 * kernels, same result) for callers that cannot allocate device memory at call time (a host
 * whose allocator is out of reach of the FFI, or a runtime that forbids allocation after
 * start-up): instead of a caller workspace it uses a fixed scratch array of
 * OC_B200_NOALLOC_SCRATCH_BYTES built into this library, one per device, for the gathered
 * activations of act-order layers, the split-K partial sums and the per-column tickets.
 *   - The first call on a device sets the scratch up (looks up its address, zeroes the
 *     tickets, waits for the device); make that first call before any stream capture.
 *   - Calls needing more scratch than that (large M * N with many splits, or a large act-order
 *     gather) fail with OC_ERR_INVALID and a message giving the bytes needed; M > 16 fails too.
 *   - Calls on one device share the scratch: two calls that overlap in time (different
 *     streams, or host threads without ordering) race and give wrong results. Order them on
 *     one stream. */
#define OC_B200_NOALLOC_SCRATCH_BYTES (8u << 20)
int oc_b200_gptq_gemv_noalloc(const oc_b200_layer* layer, const void* a, int a_dtype, int64_t M, int64_t lda,
                              const void* bias, int bias_dtype, void* c, int64_t ldc, oc_stream_t stream);

/* ---- row-packed int4/int2 linears: RTN nibble layers, DSV4 layers, expert groups ---- */
/* Device bytes the caller provides (256-byte aligned) to describe E row-packed matrices. */
size_t oc_b200_rows_table_bytes(int E);
/* Describes E row-packed weight matrices of one shape [N, K] (E = 1: a dense layer). Replaces
 * the module state of PackedRTNLinear (packed_linear.py:22-45) and Dsv4PackedLinear
 * (dsv4_packed_linear.py:59-83) and, for E > 1, the routed-expert set of the DSV4 adapter
 * (models/dsv4/loader.py:109-119).
 *   packed[e]      host array of device pointers: uint8 [N, ld_bytes], 8/wbits codes per byte,
 *                  code j of a byte at bits j*wbits (RTN: low nibble = even k)
 *   scales[e], zeros[e]  host arrays of device pointers; element (n, g) at n*stride_n + g*stride_g
 *   groupsize      k per scale group (>= K: one group per row)
 *   Scales / zeros stored group-major (stride_n == 1, stride_g >= N, rows 16-byte aligned) are staged
 *   by TMA with each 64-k weight block when a block's group rows fit 512 bytes per tensor (16-bit
 *   with groups of >= 32 k, fp32 with groups of >= 64 k, or one group per row); other layouts are
 *   read with cached global loads. Results are identical either way.
 *   mode           0: (q - z) * s in fp32, one rounding (DSV4, dsv4_packed_linear.py:52-56)
 *                  1: RTN, two roundings in the activation dtype (quant_utils.py:91-103)
 *   table          caller-allocated device memory of oc_b200_rows_table_bytes(E) bytes; the call
 *                  fills it (TMA descriptors + pointer arrays) and synchronises `stream`. */
int oc_b200_rows_layer_create(int E, const uint8_t* const* packed, int64_t ld_bytes, int wbits,
                              const void* const* scales, int scales_dtype, const void* const* zeros, int zeros_dtype,
                              int64_t stride_n, int64_t stride_g, int groupsize, int K, int N, int mode, void* table,
                              oc_stream_t stream, oc_b200_layer** out);
/* Dense (offsets == NULL): C[M, N] = A[M, K] @ W^T + bias. Grouped (offsets: device int32 [E+1]):
 * the rows of A are sorted by expert and C row r = A row r @ W_e^T for offsets[e] <= r < offsets[e+1]
 * (no bias). fp32 accumulation, one rounding to a_dtype. No workspace. */
int oc_b200_rows_gemm(const oc_b200_layer* layer, const void* a, int a_dtype, int64_t M, int64_t lda,
                      const int32_t* offsets, const void* bias, int bias_dtype, void* c, int64_t ldc,
                      oc_stream_t stream);
/* The gate and up projections of a SwiGLU expert FFN in one launch. `layer` describes [F, 2K]
 * matrices whose row n is gate row n followed by up row n (packed codes concatenated along k;
 * scale/zero groups: the K/groupsize gate groups, then the up groups), with K a multiple of 64
 * and of the groupsize. A is [M, K] (dense or grouped as in oc_b200_rows_gemm, no bias) and
 * C[M, F] = RNE(silu(g) * u), g and u each rounded to a_dtype first: the same bits as
 * oc_b200_rows_gemm on the gate and up matrices followed by oc_b200_silu_mul.
 * Replaces the first two expert matmuls and the activation of the reference's routed-expert
 * path (dsv4_packed_linear.py:95-98 per expert, models/dsv4/loader.py:92-119). */
int oc_b200_rows_gemm_swiglu(const oc_b200_layer* layer, const void* a, int a_dtype, int64_t M, int64_t lda,
                             const int32_t* offsets, void* c, int64_t ldc, oc_stream_t stream);

/* ---- packed-expert MoE -------------------------------- */
/* The reference routes in an unvendored model file (models/dsv4/loader.py:50-53);
 * the convention implemented: fp32 softmax over E logits, top-k with ties to the
 * lower expert id, weights renormalised to sum 1 when renorm != 0.
 * logits [T, E] (f32/bf16/f16) -> ids int32 [T, k], weights f32 [T, k]. E <= 1024, k <= 16. */
int oc_b200_moe_route(const void* logits, int logits_dtype, int T, int E, int k, int renorm, int32_t* ids,
                      float* weights, oc_stream_t stream);
/* Stable expert-major order of the T*k assignments: counts int32 [E],
 * offsets int32 [E+1], sorted_token int32 [T*k], slot_pos int32 [T*k]
 * (sorted position of assignment t*k+j). Replaces the per-expert loop over
 * Dsv4PackedLinear (dsv4_packed_linear.py:95-98). */
int oc_b200_moe_permute(const int32_t* ids, int T, int k, int E, int32_t* counts, int32_t* offsets,
                        int32_t* sorted_token, int32_t* slot_pos, oc_stream_t stream);
/* dst[p, :] = src[idx[p], :] for 16-bit rows of H elements (H % 8 == 0, 16-byte aligned rows). */
int oc_b200_gather_rows(const void* src, int64_t lds, const int32_t* idx, int P, int H, void* dst, int64_t ldd,
                        oc_stream_t stream);
/* h = silu(g) * u elementwise ([P, F], 16-bit, fp32 math, one rounding). */
int oc_b200_silu_mul(const void* g, const void* u, int64_t ld_in, int P, int F, void* h, int64_t ld_out, int dtype,
                     oc_stream_t stream);
/* out[t, :] = sum_j w[t,j] * y[slot_pos[t*k+j], :] (+ shared[t, :]); fp32 sum, one rounding. */
int oc_b200_moe_combine(const void* y, int64_t ldy, const int32_t* slot_pos, const float* w, int T, int k, int H,
                        const void* shared, int64_t lds, void* out, int64_t ldo, int dtype, oc_stream_t stream);

/* ---- Conv1d as a GEMM ------------------------------------------------------
 * a[(b T + t) lda + c ksize + k] = x[b, c, t stride + k dilation - pad] (0 outside the input),
 * 16-bit values, x element (b, c, l) at b sxb + c sxc + l; columns C ksize .. cols_out - 1 are 0.
 * With the RTN nibble table of a Conv1d weight [out, C ksize] it turns PackedInt4Conv1d.forward
 * (reference packed_conv.py:123-170: dequant + F.conv1d) into oc_b200_rows_gemm. */
int oc_b200_im2col_1d(const void* x, int64_t sxb, int64_t sxc, int B, int C, int L, int ksize, int stride,
                      int dilation, int pad, int T, int cols_out, void* a, int64_t lda, oc_stream_t stream);

/* ---- tensor-parallel reduction ---------------------------------------------
 * Sum over the `world` ranks of a job of n_elems bf16 values (n_elems % 8 == 0) held in one NVLink
 * multicast object, in place: afterwards every rank's copy holds the sum as the NVLink switch adds
 * bf16 (within one bf16 ulp of the exact sum; not always the nearest value). mc_ptr is the multicast address of the first element (16-byte aligned).
 * flags_dev points to a device array of `world` pointers, one per rank, to that rank's flag array
 * of at least 2 * blocks * world zero-initialised uint32 words visible to every rank (symmetric
 * memory); `epoch` must grow by at least one with every call on the same flag arrays, and every
 * rank makes the same calls in the same order with the same `blocks` (1..64). Stream-ordered; a
 * rank that does not arrive within the wait bound (OC_OPT_WAIT_US, default 2 s) makes the kernel
 * record a device error (oc_b200_read_device_error) and return without writing.
 * No reference counterpart (the reference has no distributed code); it replaces the NCCL
 * all-reduce after each row-parallel linear of the tensor-parallel DiT stack. */
int oc_b200_nvls_allreduce_bf16(void* mc_ptr, int64_t n_elems, void* const* flags_dev, int rank, int world,
                                uint32_t epoch, int blocks, oc_stream_t stream);

/* The same sum followed by an RMS norm of every row, in place: `rows` rows of `cols` bf16 values
 * (cols a multiple of 8, at most 4096; rows stored contiguously from mc_ptr). Afterwards every
 * rank's copy holds y = bf16(s * rsqrt(mean(s^2) + eps) * gain) per row, s the switch's bf16 sum
 * of the ranks' rows (as oc_b200_nvls_allreduce_bf16 leaves it), the mean square taken in fp32;
 * gain is an optional [cols] bf16 vector (16-byte aligned; NULL: no gain). The ranks split the
 * rows, so each row is normalized once in the job instead of once per rank. Flags, epoch, blocks,
 * ordering and the bounded waits are those of oc_b200_nvls_allreduce_bf16, whose flag arrays and
 * epoch sequence it shares.
 * No reference counterpart; it replaces the NCCL all-reduce and the norm that follows it in
 * the tensor-parallel DiT block. */
int oc_b200_nvls_allreduce_rmsnorm_bf16(void* mc_ptr, int rows, int cols, const void* gain, float eps,
                                        void* const* flags_dev, int rank, int world, uint32_t epoch, int blocks,
                                        oc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* OC_B200_H_ */
