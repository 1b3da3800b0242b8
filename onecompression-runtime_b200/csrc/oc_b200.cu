// C ABI of the onecomp B200 hot path: argument checks, launch configuration,
// TMA descriptors and kernel dispatch. One translation unit (no -rdc).
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/oc_b200.h"
#include "common.cuh"
#include "dequant.cuh"
#include "gemm_rows.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "gemv_tma.cuh"
#include "gemv_tc.cuh"
#include "gemv_sk.cuh"
#include "gemv_i8.cuh"
#include "allreduce.cuh"
#include "moe.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return OC_OK;
  return fail(OC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int launch_check(const char* what) { return cuda_check(cudaGetLastError(), what); }

bool dt16(int dt) { return dt == OC_DT_F16 || dt == OC_DT_BF16; }
bool dtf(int dt) { return dt == OC_DT_F16 || dt == OC_DT_BF16 || dt == OC_DT_F32; }
bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

std::atomic<int> g_opt_path{0}, g_opt_tile{0}, g_opt_gemv_ctas{2}, g_opt_gemv_impl{4}, g_opt_tc_pair{1};
// failure tests only: bound of the decode GEMV's pipeline waits (0: OC_WAIT_NS) and the stage its
// first CTA leaves unissued (0: none)
std::atomic<int> g_opt_wait_us{0}, g_opt_test_stall{0};
// persistent tcgen05 GEMMs: at most this many CTAs (0: one per SM), leaving SMs to a collective
// that runs beside them
std::atomic<int> g_opt_tc_max_ctas{0};
std::atomic<int> g_opt_gemv_prep{1};

constexpr int kMaxDevices = 64;
// Tickets at the head of every GEMV workspace, zero between launches (each launch re-arms the ones it
// takes): one per 128-column tile for the split-K kernels (at most 256 tiles), one per (256-column
// tile, consumer warp) for the stream-K kernel (at most 256 tiles x 8 warps).
constexpr size_t kTicketBytes = 8192;
constexpr int kSplitTilesMax = 256;
constexpr int kSkTilesMax = (int)(kTicketBytes / 4) / oc::kSkWarps;
int g_sm_count[kMaxDevices];
std::mutex g_mu;

int current_device(int* dev) { return cuda_check(cudaGetDevice(dev), "cudaGetDevice"); }

int sm_count(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = v > 0 ? v : 148;
  }
  return g_sm_count[dev];
}

// CTAs of a persistent tcgen05 GEMM: one per SM, or fewer under OC_OPT_TC_MAX_CTAS.
int tc_ctas(int dev) {
  const int sms = sm_count(dev);
  const int cap = g_opt_tc_max_ctas.load();
  return (cap > 0 && cap < sms) ? cap : sms;
}

// Launch with programmatic stream serialization (PDL): the kernel may start while the previous
// kernel in the stream finishes, and orders itself with griddepcontrol.wait.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char* what,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (int rc = cuda_check(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), what)) return rc;
  return launch_check(what);
}

int grid_1d(long long total, int threads, int dev) {
  long long blocks = (total + threads - 1) / threads;
  long long cap = (long long)sm_count(dev) * 16;
  if (blocks > cap) blocks = cap;
  return (int)(blocks < 1 ? 1 : blocks);
}

// ---- cuTensorMapEncodeTiled through the runtime's driver entry point -------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(OC_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (!aligned(base, 16) || row_stride_bytes % 16 != 0 || (box_inner * esize) % 16 != 0)
    return fail(OC_ERR_INVALID, "TMA operand alignment: base %p stride %llu", base,
                (unsigned long long)row_stride_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return OC_OK;
}

}  // namespace

struct oc_b200_layer {
  int kind;                // 0: AutoGPTQ layer, 1: row-packed (RTN / DSV4) layer or expert group
  int device;
  const uint32_t* qw;
  const uint32_t* qz;
  const void* s;
  int s_dtype;
  const int32_t* kperm;
  const int32_t* wgrp;
  int K_in, Kp, N, G, gs, v1;
  int sz_tma, sz_rows;     // scales/zeros staged by TMA in the tcgen05 kernel
  CUtensorMap tmap_w, tmap_s, tmap_z;
  int gt_ok, gt_rows;      // decode GEMV fed by TMA (uniform groups of 32, 64 or 128*n rows)
  CUtensorMap tmap_gw, tmap_gs, tmap_gz;
  CUtensorMap tmap_s1, tmap_z1;  // one scale / zero row per box (tcgen05 decode GEMV)
  int sk_ok;               // stream-K decode GEMV: gt_ok layouts with N >= 256
  CUtensorMap tmap_ks, tmap_kz;  // 256-column scale / zero boxes of the stream-K GEMV
  CUtensorMap tmap_kp;     // [16 word rows x 256 columns] boxes of qweight: the stream-K GEMV's L2 prefetch
  // row-packed layers
  int E, wbits, mode, s_dtype_r, z_dtype_r;
  long long stride_n, stride_g;
  const CUtensorMap* d_wmaps;
  const void* const* d_sptr;
  const void* const* d_zptr;
};

extern "C" {

int oc_b200_abi_version(void) { return 1; }

const char* oc_b200_last_error(void) { return g_last_error.c_str(); }

int oc_b200_device_check(int device) {
  int major = 0, minor = 0;
  int rc = cuda_check(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device), "capability");
  if (rc) return rc;
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0)
    return fail(OC_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200) only", device,
                major, minor);
  return OC_OK;
}

int oc_b200_set_option(int key, int value) {
  switch (key) {
    case OC_OPT_GEMM_PATH:
      if (value < 0 || value > 2) return fail(OC_ERR_INVALID, "OC_OPT_GEMM_PATH: %d", value);
      g_opt_path = value;
      return OC_OK;
    case OC_OPT_TC_TILE:
      if (value != 0 && value != 128 && value != 192 && value != 256 && value != 384 && value != 448)
        return fail(OC_ERR_INVALID, "OC_OPT_TC_TILE: %d", value);
      g_opt_tile = value;
      return OC_OK;
    case OC_OPT_GEMV_CTAS:
      if (value < 1 || value > 32) return fail(OC_ERR_INVALID, "OC_OPT_GEMV_CTAS: %d", value);
      g_opt_gemv_ctas = value;
      return OC_OK;
    case OC_OPT_TC_PAIR:
      if (value < 0 || value > 2) return fail(OC_ERR_INVALID, "OC_OPT_TC_PAIR: %d", value);
      g_opt_tc_pair = value;
      return OC_OK;
    case OC_OPT_GEMV_IMPL:
      if (value < 0 || value > 4) return fail(OC_ERR_INVALID, "OC_OPT_GEMV_IMPL: %d", value);
      g_opt_gemv_impl = value;
      return OC_OK;
    case OC_OPT_WAIT_US:
      if (value < 0) return fail(OC_ERR_INVALID, "OC_OPT_WAIT_US: %d", value);
      g_opt_wait_us = value;
      return OC_OK;
    case OC_OPT_TC_MAX_CTAS:
      if (value < 0) return fail(OC_ERR_INVALID, "OC_OPT_TC_MAX_CTAS: %d", value);
      g_opt_tc_max_ctas = value;
      return OC_OK;
    case OC_OPT_GEMV_PREP:
      if (value < 0 || value > 1) return fail(OC_ERR_INVALID, "OC_OPT_GEMV_PREP: %d", value);
      g_opt_gemv_prep = value;
      return OC_OK;
    case OC_OPT_TEST_STALL:
      if (value < 0) return fail(OC_ERR_INVALID, "OC_OPT_TEST_STALL: %d", value);
      g_opt_test_stall = value;
      return OC_OK;
  }
  return fail(OC_ERR_INVALID, "unknown option %d", key);
}

int oc_b200_get_option(int key, int* value) {
  if (!value) return fail(OC_ERR_INVALID, "get_option: value is NULL");
  switch (key) {
    case OC_OPT_GEMM_PATH: *value = g_opt_path.load(); return OC_OK;
    case OC_OPT_TC_TILE: *value = g_opt_tile.load(); return OC_OK;
    case OC_OPT_GEMV_CTAS: *value = g_opt_gemv_ctas.load(); return OC_OK;
    case OC_OPT_GEMV_IMPL: *value = g_opt_gemv_impl.load(); return OC_OK;
    case OC_OPT_TC_PAIR: *value = g_opt_tc_pair.load(); return OC_OK;
    case OC_OPT_WAIT_US: *value = g_opt_wait_us.load(); return OC_OK;
    case OC_OPT_TEST_STALL: *value = g_opt_test_stall.load(); return OC_OK;
    case OC_OPT_TC_MAX_CTAS: *value = g_opt_tc_max_ctas.load(); return OC_OK;
    case OC_OPT_GEMV_PREP: *value = g_opt_gemv_prep.load(); return OC_OK;
  }
  return fail(OC_ERR_INVALID, "unknown option %d", key);
}

int oc_b200_read_device_error(int* code, oc_stream_t stream) {
  if (!code) return fail(OC_ERR_INVALID, "code is NULL");
  unsigned v = 0, zero = 0;
  int rc = cuda_check(cudaMemcpyFromSymbolAsync(&v, oc::g_oc_dev_error, sizeof(v), 0, cudaMemcpyDeviceToHost, stream),
                      "read device error");
  if (rc) return rc;
  rc = cuda_check(cudaMemcpyToSymbolAsync(oc::g_oc_dev_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream),
                  "clear device error");
  if (rc) return rc;
  rc = cuda_check(cudaStreamSynchronize(stream), "sync");
  if (rc) return rc;
  *code = (int)v;
  return OC_OK;
}

// ---------------------------------------------------------------- Conv1d as a GEMM
int oc_b200_im2col_1d(const void* x, int64_t sxb, int64_t sxc, int B, int C, int L, int ksize, int stride,
                      int dilation, int pad, int T, int cols_out, void* a, int64_t lda, oc_stream_t stream) {
  if (!x || !a) return fail(OC_ERR_INVALID, "im2col_1d: NULL pointer");
  if (B < 0 || C <= 0 || L < 0 || ksize <= 0 || stride <= 0 || dilation <= 0 || pad < 0 || T < 0)
    return fail(OC_ERR_INVALID, "im2col_1d: B=%d C=%d L=%d k=%d stride=%d dilation=%d pad=%d T=%d", B, C, L, ksize,
                stride, dilation, pad, T);
  if (cols_out < C * ksize || lda < cols_out)
    return fail(OC_ERR_INVALID, "im2col_1d: cols_out=%d lda=%lld for %d columns", cols_out, (long long)lda,
                C * ksize);
  const long long rows = (long long)B * T;
  if (rows == 0) return OC_OK;
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  oc::im2col1d_kernel<<<grid_1d(rows * cols_out, 256, dev), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint16_t*>(x), (long long)sxb, (long long)sxc, C, L, ksize, stride, dilation, pad, T,
      cols_out, rows, reinterpret_cast<uint16_t*>(a), (long long)lda);
  return launch_check("im2col_1d");
}

// ---------------------------------------------------------------- NVLS all-reduce
int oc_b200_nvls_allreduce_bf16(void* mc_ptr, int64_t n_elems, void* const* flags_dev, int rank, int world,
                                uint32_t epoch, int blocks, oc_stream_t stream_) {
  if (!mc_ptr || !flags_dev) return fail(OC_ERR_INVALID, "nvls_allreduce: NULL pointer");
  if (n_elems < 0 || n_elems % 8 != 0 || !aligned(mc_ptr, 16))
    return fail(OC_ERR_INVALID, "nvls_allreduce: %lld elements at %p (needs 16-byte vectors)", (long long)n_elems,
                mc_ptr);
  if (world < 1 || world > oc::kArMaxWorld || rank < 0 || rank >= world)
    return fail(OC_ERR_INVALID, "nvls_allreduce: rank %d of %d (at most %d ranks)", rank, world, oc::kArMaxWorld);
  if (blocks < 1 || blocks > oc::kArMaxBlocks)
    return fail(OC_ERR_INVALID, "nvls_allreduce: blocks=%d (1..%d)", blocks, oc::kArMaxBlocks);
  if (n_elems == 0) return OC_OK;
  oc::ArParams p{};
  p.mc = reinterpret_cast<uint4*>(mc_ptr);
  p.n16 = n_elems / 8;
  p.flags = reinterpret_cast<uint32_t* const*>(flags_dev);
  p.rank = rank;
  p.world = world;
  p.epoch = epoch;
  const int wait_us = g_opt_wait_us.load();
  p.wait_ns = wait_us > 0 ? 1000ull * (unsigned long long)wait_us : (unsigned long long)OC_WAIT_NS;
  oc::nvls_allreduce_bf16_kernel<<<blocks, oc::kArThreads, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(p);
  return launch_check("nvls_allreduce_bf16");
}

int oc_b200_nvls_allreduce_rmsnorm_bf16(void* mc_ptr, int rows, int cols, const void* gain, float eps,
                                        void* const* flags_dev, int rank, int world, uint32_t epoch, int blocks,
                                        oc_stream_t stream_) {
  if (!mc_ptr || !flags_dev) return fail(OC_ERR_INVALID, "nvls_allreduce_rmsnorm: NULL pointer");
  constexpr int kMaxCols = oc::kArNormMaxVpl * 32 * 8;
  if (rows < 0 || cols < 8 || cols % 8 != 0 || cols > kMaxCols || !aligned(mc_ptr, 16) ||
      (gain && !aligned(gain, 16)))
    return fail(OC_ERR_INVALID,
                "nvls_allreduce_rmsnorm: %d x %d at %p, gain %p (cols a multiple of 8 up to %d, 16-byte aligned "
                "rows and gain)", rows, cols, mc_ptr, gain, kMaxCols);
  if (!(eps >= 0.f) || !(eps < 1e30f)) return fail(OC_ERR_INVALID, "nvls_allreduce_rmsnorm: eps=%g", (double)eps);
  if (world < 1 || world > oc::kArMaxWorld || rank < 0 || rank >= world)
    return fail(OC_ERR_INVALID, "nvls_allreduce_rmsnorm: rank %d of %d (at most %d ranks)", rank, world,
                oc::kArMaxWorld);
  if (blocks < 1 || blocks > oc::kArMaxBlocks)
    return fail(OC_ERR_INVALID, "nvls_allreduce_rmsnorm: blocks=%d (1..%d)", blocks, oc::kArMaxBlocks);
  if (rows == 0) return OC_OK;
  oc::ArNormParams p{};
  p.ar.mc = reinterpret_cast<uint4*>(mc_ptr);
  p.ar.n16 = (long long)rows * (cols / 8);
  p.ar.flags = reinterpret_cast<uint32_t* const*>(flags_dev);
  p.ar.rank = rank;
  p.ar.world = world;
  p.ar.epoch = epoch;
  const int wait_us = g_opt_wait_us.load();
  p.ar.wait_ns = wait_us > 0 ? 1000ull * (unsigned long long)wait_us : (unsigned long long)OC_WAIT_NS;
  p.rows = rows;
  p.cols = cols;
  p.gain = reinterpret_cast<const uint4*>(gain);
  p.eps = eps;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_);
  const int vpl = (cols / 8 + 31) / 32;  // 16-byte vectors per lane
  if (vpl <= 4)
    oc::nvls_allreduce_rmsnorm_bf16_kernel<4><<<blocks, oc::kArNormThreads, 0, s>>>(p);
  else if (vpl <= 8)
    oc::nvls_allreduce_rmsnorm_bf16_kernel<8><<<blocks, oc::kArNormThreads, 0, s>>>(p);
  else
    oc::nvls_allreduce_rmsnorm_bf16_kernel<16><<<blocks, oc::kArNormThreads, 0, s>>>(p);
  return launch_check("nvls_allreduce_rmsnorm_bf16");
}

// ---------------------------------------------------------------- unpack / pack / dequant
int oc_b200_gptq_unpack(const int32_t* qweight, int K, int N, int wbits, int32_t* w_int, oc_stream_t stream) {
  if (!qweight || !w_int || K <= 0 || N <= 0) return fail(OC_ERR_INVALID, "gptq_unpack: bad arguments");
  if (32 % wbits != 0) return fail(OC_ERR_INVALID, "wbits must divide 32, got %d", wbits);
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  oc::gptq_unpack_kernel<<<grid_1d((long long)K * N, 256, dev), 256, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(qweight), K, N, wbits, w_int);
  return launch_check("gptq_unpack");
}

int oc_b200_gptq_unpack_zeros(const int32_t* qzeros, int G, int N, int wbits, int32_t* zeros, oc_stream_t stream) {
  if (!qzeros || !zeros || G <= 0 || N <= 0) return fail(OC_ERR_INVALID, "gptq_unpack_zeros: bad arguments");
  if (32 % wbits != 0 || N % (32 / wbits) != 0) return fail(OC_ERR_INVALID, "unpack_zeros: wbits %d N %d", wbits, N);
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  oc::gptq_unpack_zeros_kernel<<<grid_1d((long long)G * N, 256, dev), 256, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(qzeros), G, N, wbits, zeros);
  return launch_check("gptq_unpack_zeros");
}

int oc_b200_gptq_pack(const int32_t* w_int, int N, int K, int wbits, int32_t* qweight, oc_stream_t stream) {
  if (!w_int || !qweight || K <= 0 || N <= 0) return fail(OC_ERR_INVALID, "gptq_pack: bad arguments");
  if (32 % wbits != 0) return fail(OC_ERR_INVALID, "wbits must divide 32, got %d", wbits);
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  const int rows = (K + 32 / wbits - 1) / (32 / wbits);
  oc::gptq_pack_kernel<<<grid_1d((long long)rows * N, 256, dev), 256, 0, stream>>>(
      w_int, N, K, wbits, reinterpret_cast<uint32_t*>(qweight));
  return launch_check("gptq_pack");
}

int oc_b200_gptq_dequant(const int32_t* qweight, const int32_t* qzeros, const void* scales, int scales_dtype,
                         const int64_t* g_idx, int K, int N, int G, int groupsize, int wbits, int v1, void* out,
                         int out_dtype, oc_stream_t stream) {
  if (!qweight || !qzeros || !scales || !out) return fail(OC_ERR_INVALID, "gptq_dequant: NULL pointer");
  if (K <= 0 || N <= 0 || G <= 0) return fail(OC_ERR_INVALID, "gptq_dequant: K=%d N=%d G=%d", K, N, G);
  if (wbits != 4 && wbits != 8 && wbits != 2) return fail(OC_ERR_UNSUPPORTED, "gptq_dequant: wbits=%d", wbits);
  if (N % (32 / wbits) != 0) return fail(OC_ERR_INVALID, "N=%d must be a multiple of %d", N, 32 / wbits);
  if (!g_idx && groupsize <= 0) return fail(OC_ERR_INVALID, "groupsize must be > 0 without g_idx");
  if (!dtf(scales_dtype) || !dtf(out_dtype)) return fail(OC_ERR_INVALID, "gptq_dequant: dtype");
  const int pf = 32 / wbits;
  if (out_dtype == OC_DT_F32) {
    int dev = 0;
    if (int rc = current_device(&dev)) return rc;
    oc::gptq_dequant_f32_kernel<<<grid_1d((long long)N * K, 256, dev), 256, 0, stream>>>(
        reinterpret_cast<const uint32_t*>(qweight), reinterpret_cast<const uint32_t*>(qzeros), scales, scales_dtype,
        reinterpret_cast<const long long*>(g_idx), K, N, groupsize, wbits, v1, reinterpret_cast<float*>(out));
    return launch_check("gptq_dequant_f32");
  }
  dim3 grid((N + 31) / 32, ((K + pf - 1) / pf + 7) / 8);
  const auto* qw = reinterpret_cast<const uint32_t*>(qweight);
  const auto* qz = reinterpret_cast<const uint32_t*>(qzeros);
  auto* o = reinterpret_cast<uint16_t*>(out);
  const auto* gi = reinterpret_cast<const long long*>(g_idx);
  if (wbits == 4)
    oc::gptq_dequant_kernel<4><<<grid, 256, 0, stream>>>(qw, qz, scales, scales_dtype, gi, K, N, G, groupsize, v1, o,
                                                         out_dtype);
  else if (wbits == 8)
    oc::gptq_dequant_kernel<8><<<grid, 256, 0, stream>>>(qw, qz, scales, scales_dtype, gi, K, N, G, groupsize, v1, o,
                                                         out_dtype);
  else
    oc::gptq_dequant_kernel<2><<<grid, 256, 0, stream>>>(qw, qz, scales, scales_dtype, gi, K, N, G, groupsize, v1, o,
                                                         out_dtype);
  return launch_check("gptq_dequant");
}

int oc_b200_rtn_dequant(const uint8_t* qweight_u8, int64_t ld_bytes, const void* scales, int scales_dtype,
                        const void* zeros, int zeros_dtype, int K, int N, int G, void* out, int out_dtype,
                        oc_stream_t stream) {
  if (!qweight_u8 || !scales || !zeros || !out) return fail(OC_ERR_INVALID, "rtn_dequant: NULL pointer");
  if (K <= 0 || N <= 0 || G <= 0 || ld_bytes * 2 < K) return fail(OC_ERR_INVALID, "rtn_dequant: shape");
  if (G != 1 && K % G != 0)
    return fail(OC_ERR_INVALID, "in_features=%d not divisible by num_groups=%d", K, G);
  if (!dtf(scales_dtype) || !dtf(zeros_dtype) || !dtf(out_dtype)) return fail(OC_ERR_INVALID, "rtn_dequant: dtype");
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  oc::rtn_dequant_kernel<<<grid_1d((long long)N * K, 256, dev), 256, 0, stream>>>(
      qweight_u8, ld_bytes, scales, scales_dtype, zeros, zeros_dtype, K, N, G, out, out_dtype);
  return launch_check("rtn_dequant");
}

int oc_b200_rtn_embedding(const int64_t* ids, int64_t n_ids, int64_t vocab, const uint8_t* qweight_u8,
                          int64_t ld_bytes, const void* scales, int scales_dtype, const void* zeros, int zeros_dtype,
                          int dim, int G, void* out, int out_dtype, oc_stream_t stream) {
  if (n_ids < 0 || vocab <= 0 || dim <= 0 || G <= 0 || ld_bytes * 2 < dim)
    return fail(OC_ERR_INVALID, "rtn_embedding: shape");
  if (n_ids == 0) return OC_OK;
  if (!ids || !qweight_u8 || !scales || !zeros || !out) return fail(OC_ERR_INVALID, "rtn_embedding: NULL pointer");
  if (G != 1 && dim % G != 0)
    return fail(OC_ERR_INVALID, "in_features=%d not divisible by num_groups=%d", dim, G);
  if (!dtf(scales_dtype) || !dtf(zeros_dtype) || !dtf(out_dtype)) return fail(OC_ERR_INVALID, "rtn_embedding: dtype");
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  oc::rtn_embedding_kernel<<<grid_1d((long long)n_ids * dim, 256, dev), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      ids, n_ids, vocab, qweight_u8, ld_bytes, scales, scales_dtype, zeros, zeros_dtype, dim, G, out, out_dtype);
  return launch_check("rtn_embedding");
}

int oc_b200_dsv4_dequant(const uint8_t* packed, int64_t ld_bytes, int wbits, const void* scales, int scales_dtype,
                         const void* zeros, int zeros_dtype, int64_t stride_n, int64_t stride_g, int groupsize,
                         int K, int N, void* out, int out_dtype, oc_stream_t stream) {
  if (!packed || !scales || !zeros || !out) return fail(OC_ERR_INVALID, "dsv4_dequant: NULL pointer");
  if (wbits != 2 && wbits != 4 && wbits != 8) return fail(OC_ERR_UNSUPPORTED, "dsv4_dequant: wbits=%d", wbits);
  if (K <= 0 || N <= 0 || ld_bytes * (8 / wbits) < K) return fail(OC_ERR_INVALID, "dsv4_dequant: shape");
  if (!dtf(scales_dtype) || !dtf(zeros_dtype) || !dt16(out_dtype)) return fail(OC_ERR_INVALID, "dsv4_dequant: dtype");
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  oc::dsv4_dequant_kernel<<<grid_1d((long long)N * K, 256, dev), 256, 0, stream>>>(
      packed, ld_bytes, wbits, scales, scales_dtype, zeros, zeros_dtype, stride_n, stride_g, groupsize, K, N,
      reinterpret_cast<uint16_t*>(out), out_dtype);
  return launch_check("dsv4_dequant");
}

int oc_b200_gptq_repack_k(const int32_t* qweight, const int32_t* k_perm, int k_packed, int N, int32_t* qweight_out,
                          oc_stream_t stream) {
  if (!qweight || !k_perm || !qweight_out) return fail(OC_ERR_INVALID, "repack_k: NULL pointer");
  if (k_packed <= 0 || k_packed % 8 != 0 || N <= 0) return fail(OC_ERR_INVALID, "repack_k: k_packed=%d", k_packed);
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  oc::gptq_repack_k_kernel<<<grid_1d((long long)(k_packed / 8) * N, 256, dev), 256, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(qweight), k_perm, k_packed, N, reinterpret_cast<uint32_t*>(qweight_out));
  return launch_check("repack_k");
}

int oc_b200_gptq_repack_k_ex(const int32_t* qweight, const int32_t* k_perm, int k_packed, int N, int wbits,
                             int32_t* qweight_out, oc_stream_t stream) {
  if (wbits == 4) return oc_b200_gptq_repack_k(qweight, k_perm, k_packed, N, qweight_out, stream);
  if (wbits != 8) return fail(OC_ERR_UNSUPPORTED, "repack_k: wbits=%d (4 or 8)", wbits);
  if (!qweight || !k_perm || !qweight_out) return fail(OC_ERR_INVALID, "repack_k: NULL pointer");
  if (k_packed <= 0 || k_packed % 4 != 0 || N <= 0) return fail(OC_ERR_INVALID, "repack_k: k_packed=%d", k_packed);
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  oc::gptq_repack_k8_kernel<<<grid_1d((long long)(k_packed / 4) * N, 256, dev), 256, 0,
                              reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(qweight), k_perm, k_packed, N, reinterpret_cast<uint32_t*>(qweight_out));
  return launch_check("repack_k8");
}

int oc_b200_permute_cols(const void* x, int64_t ldx, int64_t M, int K, const int32_t* k_perm, int k_packed,
                         void* x_out, oc_stream_t stream) {
  if (!x || !k_perm || !x_out || M < 0 || K <= 0 || k_packed <= 0) return fail(OC_ERR_INVALID, "permute_cols");
  if (M == 0) return OC_OK;
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  return launch_pdl(oc::permute_cols_kernel, dim3(grid_1d(M * k_packed, 256, dev)), dim3(256), 0, stream,
                    "permute_cols", reinterpret_cast<const uint16_t*>(x), (long long)ldx, (int)M, K, k_perm, k_packed,
                    reinterpret_cast<uint16_t*>(x_out));
}

// ---------------------------------------------------------------- GPTQ layer
// 8-bit layers: uniform groups in the kernel's K order. An act-order layer whose groups all hold
// groupsize rows (a permutation of k // groupsize) is uniform once its rows are sorted by group:
// k_perm (kernel row -> source row, in_features entries) gathers the activation columns and
// qweight is the repacked copy (oc_b200_gptq_repack_k_ex).
static int gptq_layer_create8(const int32_t* qweight, const int32_t* qzeros, const void* scales, int scales_dtype,
                              const int32_t* k_perm, int in_features, int N, int G, int groupsize, int v1,
                              oc_b200_layer** out) {
  const int ks = oc::gt_stage_k<8>();
  if (in_features < ks || in_features % 8 != 0)
    return fail(OC_ERR_UNSUPPORTED, "layer_create: 8-bit in_features=%d (needs a multiple of 8, >= %d)", in_features,
                ks);
  if (N < oc::kGemvCols || N % 32 != 0)
    return fail(OC_ERR_UNSUPPORTED, "layer_create: 8-bit N=%d (needs a multiple of 32, >= %d)", N, oc::kGemvCols);
  if (groupsize != 32 && (groupsize <= 0 || groupsize % ks != 0))
    return fail(OC_ERR_UNSUPPORTED, "layer_create: 8-bit groupsize=%d (needs 32 or a multiple of %d)", groupsize, ks);
  if (G != (in_features + groupsize - 1) / groupsize)
    return fail(OC_ERR_INVALID, "layer_create: G=%d for in_features=%d groupsize=%d", G, in_features, groupsize);
  if (!aligned(qweight, 16) || !aligned(scales, 16) || !aligned(qzeros, 16))
    return fail(OC_ERR_UNSUPPORTED, "layer_create: 8-bit tensors must be 16-byte aligned");
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (int rc = oc_b200_device_check(dev)) return rc;
  auto* L = new oc_b200_layer();
  L->kind = 0;
  L->wbits = 8;
  L->device = dev;
  L->qw = reinterpret_cast<const uint32_t*>(qweight);
  L->qz = reinterpret_cast<const uint32_t*>(qzeros);
  L->s = scales;
  L->s_dtype = scales_dtype;
  L->K_in = in_features;
  L->Kp = in_features;
  L->kperm = k_perm;
  L->N = N;
  L->G = G;
  L->gs = groupsize;
  L->v1 = v1 ? 1 : 0;
  const int rows = groupsize >= ks ? 1 : ks / groupsize;
  // tcgen05 GEMM (M > 16): 16 word rows (64 k) per stage, scale / zero rows of the 64-k block
  L->sz_tma = 1;
  L->sz_rows = groupsize == 32 ? 2 : 1;
  int rc = make_tmap_2d(&L->tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qweight, (uint64_t)N,
                        (uint64_t)(in_features / 4), (uint64_t)N * 4, oc::kTcBN, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = make_tmap_2d(&L->tmap_s, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, scales, (uint64_t)N, (uint64_t)G, (uint64_t)N * 2,
                      oc::kTcBN, L->sz_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = make_tmap_2d(&L->tmap_z, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qzeros, (uint64_t)(N / 4), (uint64_t)G,
                      (uint64_t)(N / 4) * 4, oc::kTcBN / 4, L->sz_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = make_tmap_2d(&L->tmap_gw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qweight, (uint64_t)N,
                      (uint64_t)(in_features / 4), (uint64_t)N * 4, 32, 16, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc)
    rc = make_tmap_2d(&L->tmap_gs, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, scales, (uint64_t)N, (uint64_t)G,
                      (uint64_t)N * 2, oc::kGemvCols, rows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = make_tmap_2d(&L->tmap_gz, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qzeros, (uint64_t)(N / 4), (uint64_t)G,
                      (uint64_t)(N / 4) * 4, oc::kGemvCols / 4, rows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) {
    delete L;
    return rc;
  }
  L->gt_ok = 1;
  L->gt_rows = rows;
  *out = L;
  return OC_OK;
}

int oc_b200_gptq_layer_create(const int32_t* qweight, const int32_t* qzeros, const void* scales, int scales_dtype,
                              const int32_t* k_perm, const int32_t* word_group, int in_features, int k_packed, int N,
                              int G, int groupsize, int v1, oc_b200_layer** out) {
  return oc_b200_gptq_layer_create_ex(qweight, qzeros, scales, scales_dtype, k_perm, word_group, in_features,
                                      k_packed, N, G, groupsize, 4, v1, out);
}

int oc_b200_gptq_layer_create_ex(const int32_t* qweight, const int32_t* qzeros, const void* scales, int scales_dtype,
                                 const int32_t* k_perm, const int32_t* word_group, int in_features, int k_packed,
                                 int N, int G, int groupsize, int wbits, int v1, oc_b200_layer** out) {
  if (!out) return fail(OC_ERR_INVALID, "layer_create: out is NULL");
  *out = nullptr;
  if (!qweight || !qzeros || !scales) return fail(OC_ERR_INVALID, "layer_create: NULL tensor");
  if (wbits != 4 && wbits != 8) return fail(OC_ERR_UNSUPPORTED, "layer_create: wbits=%d (4 or 8)", wbits);
  if (wbits == 8) {
    if (!dt16(scales_dtype)) return fail(OC_ERR_UNSUPPORTED, "layer_create: scales must be f16 or bf16");
    if (word_group || k_packed != in_features)
      return fail(OC_ERR_UNSUPPORTED,
                  "layer_create: 8-bit layers take no word groups and no padded K permutation (k_packed=%d, "
                  "in_features=%d)", k_packed, in_features);
    return gptq_layer_create8(qweight, qzeros, scales, scales_dtype, k_perm, in_features, N, G, groupsize, v1, out);
  }
  if (!dt16(scales_dtype)) return fail(OC_ERR_UNSUPPORTED, "layer_create: scales must be f16 or bf16");
  if (in_features <= 0 || k_packed <= 0 || k_packed % 8 != 0)
    return fail(OC_ERR_INVALID, "layer_create: in_features=%d k_packed=%d (k_packed must be a multiple of 8)",
                in_features, k_packed);
  if (!k_perm && k_packed != in_features)
    return fail(OC_ERR_INVALID, "layer_create: k_packed != in_features needs k_perm");
  if (N <= 0 || N % 8 != 0) return fail(OC_ERR_INVALID, "layer_create: N=%d must be a multiple of 8", N);
  if (G <= 0 || (!word_group && (groupsize <= 0 || groupsize % 8 != 0)))
    return fail(OC_ERR_INVALID, "layer_create: groupsize=%d must be a positive multiple of 8 without word_group",
                groupsize);
  if (!aligned(qweight, 16) || !aligned(scales, 8) || !aligned(qzeros, 4))
    return fail(OC_ERR_INVALID, "layer_create: misaligned weight tensors");
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (int rc = oc_b200_device_check(dev)) return rc;
  auto* L = new oc_b200_layer();
  L->kind = 0;
  L->wbits = 4;
  L->device = dev;
  L->qw = reinterpret_cast<const uint32_t*>(qweight);
  L->qz = reinterpret_cast<const uint32_t*>(qzeros);
  L->s = scales;
  L->s_dtype = scales_dtype;
  L->kperm = k_perm;
  L->wgrp = word_group;
  L->K_in = in_features;
  L->Kp = k_packed;
  L->N = N;
  L->G = G;
  L->gs = groupsize;
  L->v1 = v1 ? 1 : 0;
  int rc = make_tmap_2d(&L->tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qweight, (uint64_t)N, (uint64_t)(k_packed / 8),
                        (uint64_t)N * 4, oc::kTcBN, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) {
    delete L;
    return rc;
  }
  // Uniform groups aligned to the 64-k block: stage scales/zeros with the packed tile.
  L->sz_tma = 0;
  L->sz_rows = 0;
  L->tmap_s = L->tmap_w;
  L->tmap_z = L->tmap_w;
  if (!word_group && N % 32 == 0 && (groupsize == 32 || groupsize % 64 == 0) && aligned(scales, 16) &&
      aligned(qzeros, 16)) {
    const int rows = groupsize == 32 ? 2 : 1;
    if (make_tmap_2d(&L->tmap_s, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, scales, (uint64_t)N, (uint64_t)G, (uint64_t)N * 2,
                     oc::kTcBN, rows, CU_TENSOR_MAP_SWIZZLE_NONE) == OC_OK &&
        make_tmap_2d(&L->tmap_z, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qzeros, (uint64_t)(N / 8), (uint64_t)G,
                     (uint64_t)(N / 8) * 4, oc::kTcBN / 8, rows, CU_TENSOR_MAP_SWIZZLE_NONE) == OC_OK) {
      L->sz_tma = 1;
      L->sz_rows = rows;
    } else {
      L->tmap_s = L->tmap_w;
      L->tmap_z = L->tmap_w;
    }
  }
  // Decode GEMV by TMA: uniform groups of 32, 64 or a multiple of 128 rows, at least one full
  // 128-column tile and one 128-k stage; other layouts take the cp.async GEMV kernels.
  L->gt_ok = 0;
  L->gt_rows = 0;
  if (!word_group && N % 32 == 0 && N >= 128 && k_packed >= 128 &&
      (groupsize == 32 || groupsize == 64 || groupsize % 128 == 0) && aligned(qweight, 16) && aligned(scales, 16) &&
      aligned(qzeros, 16)) {
    const int rows = groupsize >= 128 ? 1 : 128 / groupsize;
    if (make_tmap_2d(&L->tmap_gw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qweight, (uint64_t)N, (uint64_t)(k_packed / 8),
                     (uint64_t)N * 4, 32, 16, CU_TENSOR_MAP_SWIZZLE_128B) == OC_OK &&
        make_tmap_2d(&L->tmap_gs, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, scales, (uint64_t)N, (uint64_t)G, (uint64_t)N * 2,
                     oc::kGemvCols, rows, CU_TENSOR_MAP_SWIZZLE_NONE) == OC_OK &&
        make_tmap_2d(&L->tmap_gz, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qzeros, (uint64_t)(N / 8), (uint64_t)G,
                     (uint64_t)(N / 8) * 4, oc::kGemvCols / 8, rows, CU_TENSOR_MAP_SWIZZLE_NONE) == OC_OK &&
        make_tmap_2d(&L->tmap_s1, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, scales, (uint64_t)N, (uint64_t)G, (uint64_t)N * 2,
                     oc::kGemvCols, 1, CU_TENSOR_MAP_SWIZZLE_NONE) == OC_OK &&
        make_tmap_2d(&L->tmap_z1, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qzeros, (uint64_t)(N / 8), (uint64_t)G,
                     (uint64_t)(N / 8) * 4, oc::kGemvCols / 8, 1, CU_TENSOR_MAP_SWIZZLE_NONE) == OC_OK) {
      L->gt_ok = 1;
      L->gt_rows = rows;
    }
  }
  // Stream-K decode GEMV: the same layouts, tiles of 256 columns.
  L->sk_ok = 0;
  if (L->gt_ok && N >= oc::kSkCols && N <= oc::kSkCols * kSkTilesMax && aligned(k_perm, 16) &&
      make_tmap_2d(&L->tmap_kp, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qweight, (uint64_t)N, (uint64_t)(k_packed / 8),
                   (uint64_t)N * 4, oc::kSkCols, 16, CU_TENSOR_MAP_SWIZZLE_NONE) == OC_OK &&
      make_tmap_2d(&L->tmap_ks, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, scales, (uint64_t)N, (uint64_t)G, (uint64_t)N * 2,
                   oc::kSkCols, L->gt_rows, CU_TENSOR_MAP_SWIZZLE_NONE) == OC_OK &&
      make_tmap_2d(&L->tmap_kz, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qzeros, (uint64_t)(N / 8), (uint64_t)G,
                   (uint64_t)(N / 8) * 4, oc::kSkCols / 8, L->gt_rows, CU_TENSOR_MAP_SWIZZLE_NONE) == OC_OK)
    L->sk_ok = 1;
  *out = L;
  return OC_OK;
}

int oc_b200_layer_destroy(oc_b200_layer* layer) {
  delete layer;
  return OC_OK;
}

}  // extern "C"

namespace {


struct GemvPlan {
  int splits, kstep;
};
constexpr int kI8ClusterMax = 2;

// Split-K plan: as many K splits as fit one wave of CTAs (sm_count x OC_OPT_GEMV_CTAS, two
// 100 KB cp.async-ring CTAs per SM by default) over the layer's 128-column tiles, each K-warp
// keeping at least 4 steps of 32 k.
// Which decode kernel runs for a layer: 0 tcgen05 GEMV, 1 TMA + mma.sync GEMV, 3 stream-K GEMV,
// 4 integer-MMA GEMV (the default; up to 8 tokens, 1 above) -- all for uniform groups of 32, 64 or
// 128*n rows --, 2 cp.async + mma.sync GEMV (any layout).
int gemv_impl(const oc_b200_layer* L) {
  if (L->wbits == 8) return 1;  // 8-bit layers have only the TMA GEMV
  if (!L->gt_ok) return 2;
  const int v = g_opt_gemv_impl.load();
  if (v == 3 && !L->sk_ok) return 1;
  return v;
}

// The split-K kernel that runs where the stream-K GEMV does not (the no-allocation entry point,
// which sizes its fixed scratch for the split-K kernels): the TMA GEMV in its place.
int legacy_impl(const oc_b200_layer* L) {
  const int v = gemv_impl(L);
  return (v == 3 || v == 4) ? 1 : v;
}

// The integer decode GEMV (gemv_i8.cuh) for 4-bit uniform-group layers up to 8 tokens (one token
// tile; with two the 16-bit TMA GEMV measured faster); it splits K in the TMA GEMV's 128-k stages,
// so it shares that plan.
bool use_i8(const oc_b200_layer* L, int64_t M) { return gemv_impl(L) == 4 && M <= 8; }

// Prepared activations of the integer GEMV: [M][stages][320 B].
size_t x8_bytes(const oc_b200_layer* L, int64_t M) {
  const int KB = (L->Kp + oc::kX8StageK - 1) / oc::kX8StageK;
  return ((size_t)M * KB * oc::kX8RowBytes + 255) / 256 * 256;
}

// The stream-K GEMV runs decode sizes up to 8 tokens (one token tile); larger M takes the
// split-K kernel, whose activations come by TMA from the gathered copy.
bool use_sk(const oc_b200_layer* L, int64_t M) { return gemv_impl(L) == 3 && M <= 8; }

// Stream-K plan: units of 256 columns x 128 k, an equal run per CTA, two CTAs per SM.
struct SkPlan {
  int tiles, KB, units, upc, grid;
};
SkPlan sk_plan(const oc_b200_layer* L, int dev) {
  SkPlan q;
  q.tiles = (L->N + oc::kSkCols - 1) / oc::kSkCols;
  q.KB = (L->Kp + oc::kSkBK - 1) / oc::kSkBK;
  q.units = q.tiles * q.KB;
  const int ctas = 2 * sm_count(dev);  // two CTAs (16 consumer warps) per SM
  q.upc = (q.units + ctas - 1) / ctas;
  q.grid = (q.units + q.upc - 1) / q.upc;
  return q;
}

GemvPlan gemv_plan(const oc_b200_layer* L, int dev) {
  const int n_tiles = (L->N + oc::kGemvCols - 1) / oc::kGemvCols;
  const int steps = (L->Kp + 31) / 32;
  const int target = sm_count(dev) * g_opt_gemv_ctas.load();
  if (legacy_impl(L) == 0) {  // tcgen05 GEMV: one CTA per SM, splits in 64-k blocks, at least 4 each
    const int KB = (L->Kp + oc::kVtBK - 1) / oc::kVtBK;
    int splits = sm_count(dev) / n_tiles;
    const int max_splits = KB / 4 > 0 ? KB / 4 : 1;
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    if (n_tiles > kSplitTilesMax) splits = 1;
    const int kbs = (KB + splits - 1) / splits;
    splits = (KB + kbs - 1) / kbs;
    return {splits, kbs * (oc::kVtBK / 32)};
  }
  if (legacy_impl(L) == 1) {  // TMA GEMV: splits in whole stages (128 k, 64 k for 8-bit), at least two per CTA
    const int ks = L->wbits == 8 ? oc::gt_stage_k<8>() : oc::kGtBK;
    const int KB = (L->Kp + ks - 1) / ks;
    int splits = target / n_tiles;
    const int max_splits = KB / 2 > 0 ? KB / 2 : 1;
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    if (n_tiles > kSplitTilesMax) splits = 1;
    const int kbs = (KB + splits - 1) / splits;
    splits = (KB + kbs - 1) / kbs;
    return {splits, kbs * (oc::kGtBK / 32)};
  }
  int splits = target / n_tiles;
  const int max_splits = steps / 8 > 0 ? steps / 8 : 1;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  if (n_tiles > kSplitTilesMax) splits = 1;
  int kstep = (steps + splits - 1) / splits;
  splits = (steps + kstep - 1) / kstep;
  return {splits, kstep};
}

// The integer GEMV splits K like the TMA GEMV (128-k stages); up to kI8ClusterMax splits of a tile
// reduce inside their thread-block cluster, more through the workspace.
bool i8_cluster(int splits) { return splits > 1 && splits <= kI8ClusterMax; }

// The integer GEMV prepares its activations inside the GEMV (no preparation launch, no workspace
// copy) for one token when the layer has no K permutation and a K split spans at most
// kPrepMaxStages stages. Measured per layer on the config-2 shapes (B200, CUDA graph of copies
// of one layer): M = 1 without act-order 0.3-1.4 us faster; with act-order every CTA would gather
// its split's activation columns with scattered 2-byte loads (hundreds of CTAs, the same columns)
// and the down layer ran 3 us slower (7 us at M = 2); at M = 2 without act-order mixed
// (-1.4 to +1.0 us). Those cases keep the preparation launch.
bool i8_prep(int64_t M, int kb_per_split, bool has_kperm) {
  return g_opt_gemv_prep.load() != 0 && M == 1 && !has_kperm && kb_per_split <= oc::kPrepMaxStages;
}

// Tokens per tcgen05 tile when the caller leaves it to the library: the preset with the
// least (waves of persistent CTAs) x (measured time of one tile at K = 3072 on B200, us).
// 384 and 448 are two sub-tiles of 192 / 224 tokens sharing each dequantized weight stage.
int choose_tile(int64_t M, int n_tiles_n, int sms) {
  static const int kBt[5] = {384, 448, 256, 192, 128};
  static const double kTileUs[5] = {41.7, 42.5, 31.7, 25.0, 22.7};
  int best = 384;
  double best_cost = 1e300;
  for (int i = 0; i < 5; ++i) {
    const int64_t tiles = (int64_t)n_tiles_n * ((M + kBt[i] - 1) / kBt[i]);
    const double cost = (double)((tiles + sms - 1) / sms) * kTileUs[i];
    if (cost < best_cost) {
      best_cost = cost;
      best = kBt[i];
    }
  }
  return best;
}

// CTA pairs for the tcgen05 GEMM: 1 single CTAs (default, measured faster), 2 pairs, 0 auto
// (pairs for tiles of 256 tokens and more).
bool use_pairs(int64_t M, int bt) {
  const int v = g_opt_tc_pair.load();
  if (v == 2) return true;
  if (v == 1) return false;
  return M >= 256 && bt >= 256;
}

bool use_gemv(int64_t M) {
  const int path = g_opt_path.load();
  if (path == 1) return M <= 16;
  if (path == 2) return false;
  return M <= 16;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool layer_gemv(const oc_b200_layer* L, int64_t M) { return use_gemv(M); }

}  // namespace

extern "C" size_t oc_b200_gptq_gemm_workspace(const oc_b200_layer* L, int64_t M) {
  if (!L || M <= 0) return kTicketBytes;
  size_t bytes = kTicketBytes;
  if (layer_gemv(L, M) && use_sk(L, M)) {  // gathers its own activations
    const SkPlan q = sk_plan(L, L->device);
    if (q.grid > 1) bytes += align_up((size_t)(q.tiles + q.grid) * M * oc::kSkCols * 4, 256);
    return bytes;
  }
  if (layer_gemv(L, M) && use_i8(L, M)) {  // prepared activations (the act-order gather included)
    bytes += x8_bytes(L, M);
    const GemvPlan gp = gemv_plan(L, L->device);
    if (gp.splits > 1 && !i8_cluster(gp.splits)) bytes += align_up((size_t)gp.splits * M * L->N * 4, 256);
    return bytes;
  }
  if (L->kperm) bytes += align_up((size_t)M * L->Kp * 2, 256);  // gathered activations
  if (layer_gemv(L, M)) {
    const GemvPlan gp = gemv_plan(L, L->device);
    if (gp.splits > 1) bytes += align_up((size_t)gp.splits * M * L->N * 4, 256);
  }
  return bytes;
}

namespace {

// Launch one GEMV kernel with its cp.async ring as dynamic shared memory (the attribute is
// set once per device for each kernel: one template instance per kernel).
template <auto Kern>
int launch_gemv_k(int smem, const oc::GemvParams& p, dim3 grid, cudaStream_t stream, const char* what) {
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = cuda_check(cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                            "cudaFuncSetAttribute(gemv smem)"))
      return rc;
    attr_set[dev] = true;
  }
  Kern<<<grid, oc::kGemvThreads, smem, stream>>>(p);
  return launch_check(what);
}

template <auto Kern>
int launch_gt_k(int smem, dim3 grid, cudaStream_t stream, const oc_b200_layer* L, const CUtensorMap& tx,
                const oc::GtParams& g) {
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = cuda_check(cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                            "cudaFuncSetAttribute(gemv tma smem)"))
      return rc;
    attr_set[dev] = true;
  }
  return launch_pdl(Kern, grid, dim3(oc::kGtThreads), (size_t)smem, stream, "gptq_gemv_tma", L->tmap_gw, L->tmap_gs,
                    L->tmap_gz, tx, g);
}

// The tcgen05 decode GEMV (layers with gt_ok); the activation tensor map is made per call.
template <bool BF16>
int launch_gemv_tcv(const oc_b200_layer* L, const oc::GemvParams& p, const GemvPlan& gp, int n_tiles,
                    cudaStream_t stream) {
  oc::VtParams v{};
  v.g = p;
  v.kb_per_split = gp.kstep / (oc::kVtBK / 32);
  CUtensorMap tx;
  if (int rc = make_tmap_2d(&tx, BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.x,
                            (uint64_t)p.Kp, (uint64_t)p.M, (uint64_t)p.ldx * 2, oc::kVtBK, (uint32_t)oc::kVtN,
                            CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  auto kern = oc::gptq_gemv_tc_kernel<BF16>;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, oc::kVtSmemBytes),
                            "cudaFuncSetAttribute(gemv tc smem)"))
      return rc;
    attr_set[dev] = true;
  }
  return launch_pdl(kern, dim3(n_tiles, gp.splits), dim3(oc::kVtThreads), (size_t)oc::kVtSmemBytes, stream,
                    "gptq_gemv_tc", L->tmap_w, L->tmap_s1, L->tmap_z1, tx, v);
}

// The TMA-fed factored GEMV (layers with gt_ok); the activation tensor map is made per call.
template <bool BF16>
int launch_gemv_tma(const oc_b200_layer* L, const oc::GemvParams& p, const GemvPlan& gp, int n_tiles,
                    cudaStream_t stream) {
  oc::GtParams g{};
  g.g = p;
  const int ks = L->wbits == 8 ? oc::gt_stage_k<8>() : oc::kGtBK;  // k per stage
  g.rows_sz = L->gt_rows;
  g.kb_per_split = gp.kstep / (oc::kGtBK / 32);
  const int wait_us = g_opt_wait_us.load();
  g.wait_ns = wait_us > 0 ? 1000ull * (unsigned long long)wait_us : (unsigned long long)OC_WAIT_NS;
  g.stall_stage = g_opt_test_stall.load();
  const int mt = p.M <= 8 ? 1 : 2;
  CUtensorMap tx;
  if (int rc = make_tmap_2d(&tx, BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.x,
                            (uint64_t)p.Kp, (uint64_t)p.M, (uint64_t)p.ldx * 2, (uint32_t)ks, (uint32_t)(8 * mt),
                            CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  const dim3 grid(n_tiles, gp.splits);
  if (L->wbits == 8) {
    if (mt == 1)
      return launch_gt_k<oc::gptq_gemv_tma_kernel<BF16, 1, 8>>(oc::GtCfg<1>::kSmemBytes, grid, stream, L, tx, g);
    return launch_gt_k<oc::gptq_gemv_tma_kernel<BF16, 2, 8>>(oc::GtCfg<2>::kSmemBytes, grid, stream, L, tx, g);
  }
  if (mt == 1)
    return launch_gt_k<oc::gptq_gemv_tma_kernel<BF16, 1>>(oc::GtCfg<1>::kSmemBytes, grid, stream, L, tx, g);
  return launch_gt_k<oc::gptq_gemv_tma_kernel<BF16, 2>>(oc::GtCfg<2>::kSmemBytes, grid, stream, L, tx, g);
}

// The integer decode GEMV: x8_prepare_kernel (gather + fixed-point digits into `xd`), then the
// GEMV over them; both launched with programmatic stream serialization.
template <auto Kern>
int launch_g8_k(int smem, dim3 grid, cudaStream_t stream, const oc_b200_layer* L, const CUtensorMap& tx,
                const oc::GtParams& g, int smem_extra = 0) {
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    std::lock_guard<std::mutex> lk(g_mu);
    // the largest size any launch of this kernel asks for (PREP adds the prepared stages)
    const int most = smem + (smem_extra ? oc::kPrepMaxStages * 2 * oc::kX8RowBytes : 0);
    if (int rc = cuda_check(cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, most),
                            "cudaFuncSetAttribute(gemv i8 smem)"))
      return rc;
    attr_set[dev] = true;
  }
  // with g.cluster: one cluster per column tile, its K splits
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(oc::kGtThreads);
  cfg.dynamicSmemBytes = (size_t)(smem + smem_extra);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = grid.y;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g.cluster ? 2 : 1;
  if (int rc = cuda_check(cudaLaunchKernelEx(&cfg, Kern, L->tmap_gw, L->tmap_gs, L->tmap_gz, tx, g), "gptq_gemv_i8"))
    return rc;
  return launch_check("gptq_gemv_i8");
}

template <bool BF16, int MT, bool ODD, int XR>
int launch_g8_sps(const oc_b200_layer* L, dim3 grid, cudaStream_t stream, const CUtensorMap& tx,
                  const oc::GtParams& g) {
  if (g.k_in > 0) {  // PREP: the CTAs prepare their activations (M <= 2)
    if constexpr (MT == 1 && XR == 2) {
      const int extra = g.kb_per_split * 2 * oc::kX8RowBytes;
      if (L->gt_rows == 4)
        return launch_g8_k<oc::gptq_gemv_i8_kernel<BF16, 1, 4, ODD, 2, true>>(oc::G8Cfg<1, 4, 2, true>::kSmemBytes,
                                                                              grid, stream, L, tx, g, extra);
      if (L->gt_rows == 2)
        return launch_g8_k<oc::gptq_gemv_i8_kernel<BF16, 1, 2, ODD, 2, true>>(oc::G8Cfg<1, 2, 2, true>::kSmemBytes,
                                                                              grid, stream, L, tx, g, extra);
      return launch_g8_k<oc::gptq_gemv_i8_kernel<BF16, 1, 1, ODD, 2, true>>(oc::G8Cfg<1, 1, 2, true>::kSmemBytes,
                                                                            grid, stream, L, tx, g, extra);
    }
    return fail(OC_ERR_UNSUPPORTED, "gemv_i8: activation preparation in the GEMV needs M <= 2");
  }
  if (L->gt_rows == 4)
    return launch_g8_k<oc::gptq_gemv_i8_kernel<BF16, MT, 4, ODD, XR>>(oc::G8Cfg<MT, 4, XR>::kSmemBytes, grid, stream,
                                                                      L, tx, g);
  if (L->gt_rows == 2)
    return launch_g8_k<oc::gptq_gemv_i8_kernel<BF16, MT, 2, ODD, XR>>(oc::G8Cfg<MT, 2, XR>::kSmemBytes, grid, stream,
                                                                      L, tx, g);
  return launch_g8_k<oc::gptq_gemv_i8_kernel<BF16, MT, 1, ODD, XR>>(oc::G8Cfg<MT, 1, XR>::kSmemBytes, grid, stream,
                                                                    L, tx, g);
}

template <bool BF16>
int launch_gemv_i8(const oc_b200_layer* L, const void* a, int64_t lda, const oc::GemvParams& p, const GemvPlan& gp,
                   int n_tiles, uint8_t* xd, cudaStream_t stream) {
  const int KB = (L->Kp + oc::kX8StageK - 1) / oc::kX8StageK;
  oc::GtParams g{};
  g.g = p;
  g.kb_per_split = gp.kstep / (oc::kGtBK / 32);
  if (i8_prep(p.M, g.kb_per_split, L->kperm != nullptr)) {  // each CTA prepares its split's activations
    g.g.x = reinterpret_cast<const uint16_t*>(a);
    g.g.ldx = lda;
    g.kperm = L->kperm;
    g.k_in = L->K_in;
  } else {
    const long long threads = (long long)p.M * KB * 16;
    if (int rc = launch_pdl(oc::x8_prepare_kernel<BF16>, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0,
                            stream, "x8_prepare", reinterpret_cast<const uint16_t*>(a), (long long)lda, p.M, L->K_in,
                            L->kperm, L->Kp, KB, xd))
      return rc;
  }
  g.rows_sz = L->gt_rows;
  const int wait_us = g_opt_wait_us.load();
  g.wait_ns = wait_us > 0 ? 1000ull * (unsigned long long)wait_us : (unsigned long long)OC_WAIT_NS;
  g.stall_stage = g_opt_test_stall.load();
  g.cluster = i8_cluster(gp.splits) ? 1 : 0;
  const int xr = p.M <= 2 ? 2 : (p.M <= 8 ? 8 : 16);  // activation rows per stage box
  CUtensorMap tx;
  if (int rc = make_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, xd, (uint64_t)KB * oc::kX8RowWords, (uint64_t)p.M,
                            (uint64_t)KB * oc::kX8RowBytes, (uint32_t)oc::kX8RowWords, (uint32_t)xr,
                            CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  const dim3 grid(n_tiles, gp.splits);
  if (xr == 16) return launch_g8_sps<BF16, 2, true, 16>(L, grid, stream, tx, g);
  if (xr == 8) return launch_g8_sps<BF16, 1, true, 8>(L, grid, stream, tx, g);
  if (p.M == 2) return launch_g8_sps<BF16, 1, true, 2>(L, grid, stream, tx, g);
  return launch_g8_sps<BF16, 1, false, 2>(L, grid, stream, tx, g);
}

// The stream-K decode GEMV (layers with sk_ok): activations in the caller's K order.
template <auto Kern>
int launch_sk_k(dim3 grid, cudaStream_t stream, const oc_b200_layer* L, const oc::SkParams& q) {
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = cuda_check(cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 oc::kSkSmemBytes),
                            "cudaFuncSetAttribute(gemv sk smem)"))
      return rc;
    attr_set[dev] = true;
  }
  return launch_pdl(Kern, grid, dim3(oc::kSkThreads), (size_t)oc::kSkSmemBytes, stream, "gptq_gemv_sk", L->tmap_gw,
                    L->tmap_ks, L->tmap_kz, L->tmap_kp, q);
}

template <bool BF16>
int launch_gemv_sk(const oc_b200_layer* L, const void* a, int64_t lda, int64_t M, const void* bias, int bias_dtype,
                   const void* residual, int64_t ldr, int act, void* c, int64_t ldc, float* ws, unsigned* tickets,
                   int dev, cudaStream_t stream) {
  const SkPlan pl = sk_plan(L, dev);
  oc::SkParams q{};
  q.x = reinterpret_cast<const uint16_t*>(a);
  q.ldx = lda;
  q.M = (int)M;
  q.kperm = L->kperm;
  q.K_in = L->K_in;
  q.Kp = L->Kp;
  q.N = L->N;
  q.gs = L->gs;
  q.v1 = L->v1;
  q.s_dtype = L->s_dtype;
  q.rows_sz = L->gt_rows;
  q.KB = pl.KB;
  q.units = pl.units;
  q.upc = pl.upc;
  q.bias = bias;
  q.bias_dtype = bias_dtype;
  q.residual = reinterpret_cast<const uint16_t*>(residual);
  q.ldr = ldr;
  q.act = act;
  q.out = reinterpret_cast<uint16_t*>(c);
  q.ldc = ldc;
  q.ws = ws;
  q.tickets = tickets;
  const int wait_us = g_opt_wait_us.load();
  q.wait_ns = wait_us > 0 ? 1000ull * (unsigned long long)wait_us : (unsigned long long)OC_WAIT_NS;
  q.stall_stage = g_opt_test_stall.load();
  // M <= 8: one token tile; MMA steps per scale group: 1, 2 or 4 (groups of 32, 64, >= 128 rows)
  if (L->gs == 32) return launch_sk_k<oc::gptq_gemv_sk_kernel<BF16, 1, 1>>(dim3(pl.grid), stream, L, q);
  if (L->gs == 64) return launch_sk_k<oc::gptq_gemv_sk_kernel<BF16, 1, 2>>(dim3(pl.grid), stream, L, q);
  return launch_sk_k<oc::gptq_gemv_sk_kernel<BF16, 1, 4>>(dim3(pl.grid), stream, L, q);
}

template <bool BF16, bool HAS_LO>
int launch_gemv(const oc::GemvParams& p, int n_tiles, int splits, cudaStream_t stream) {
  dim3 grid(n_tiles, splits);
  if (!p.wgrp && p.gs % 32 == 0) {  // whole groups per 32-k step: factored scaling
    if (p.M <= 8)
      return launch_gemv_k<oc::gptq_gemv_fact_kernel<BF16, 1>>(oc::GemvRing<1>::kSmemBytes, p, grid, stream,
                           "gptq_gemv_fact");
    return launch_gemv_k<oc::gptq_gemv_fact_kernel<BF16, 2>>(oc::GemvRing<2>::kSmemBytes, p, grid, stream,
                         "gptq_gemv_fact");
  }
  if (p.M <= 8)
    return launch_gemv_k<oc::gptq_gemv_kernel<BF16, HAS_LO, 1>>(oc::GemvRing<1>::kSmemBytes, p, grid, stream,
                         "gptq_gemv");
  return launch_gemv_k<oc::gptq_gemv_kernel<BF16, HAS_LO, 2>>(oc::GemvRing<2>::kSmemBytes, p, grid, stream,
                       "gptq_gemv");
}

struct TcMaps {
  CUtensorMap x, c, r;
};

template <bool BF16, bool HAS_LO, int BT, int NSUB, int ACC, int XS, int WS, int AS, int CG = 1, int WB = 4>
int launch_tc_t(const TcMaps& tm, const oc_b200_layer* L, const oc::TcParams& p, int dev, cudaStream_t stream) {
  using Cfg = oc::TcCfg<BT, NSUB, ACC, XS, WS, AS, CG, WB>;
  auto kern = oc::gptq_gemm_tc_kernel<BF16, HAS_LO, BT, NSUB, ACC, XS, WS, AS, CG, WB>;
  static bool attr_set[kMaxDevices] = {};
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes),
                            "cudaFuncSetAttribute(smem)"))
      return rc;
    attr_set[dev] = true;
  }
  if (CG == 1) {
    int grid = p.num_tiles < tc_ctas(dev) ? p.num_tiles : tc_ctas(dev);
    kern<<<grid, oc::kTcThreads, Cfg::kSmemBytes, stream>>>(tm.x, L->tmap_w, L->tmap_s, L->tmap_z, tm.c, tm.r, p);
    return launch_check("gptq_gemm_tc");
  }
  // CTA pairs: clusters of two, one pair tile (256 features) at a time
  const int pairs = tc_ctas(dev) / 2 > 0 ? tc_ctas(dev) / 2 : 1;
  const int grid = 2 * (p.num_tiles < pairs ? p.num_tiles : pairs);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(oc::kTcThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (int rc = cuda_check(cudaLaunchKernelEx(&cfg, kern, tm.x, L->tmap_w, L->tmap_s, L->tmap_z, tm.c, tm.r, p),
                          "gptq_gemm_tc (pairs)"))
    return rc;
  return launch_check("gptq_gemm_tc (pairs)");
}

// Tile presets (tokens per tile, accumulators, activation / weight / TMEM-A stages), sized to
// 512 TMEM columns and the 227 KB of shared memory with the epilogue staging tile.
template <bool BF16, bool HAS_LO>
int launch_tc(int bt, bool pair, const TcMaps& tm, const oc_b200_layer* L, const oc::TcParams& p, int dev,
              cudaStream_t stream) {
  if (L->wbits == 8) {  // 8-bit stages are twice as large: four weight stages
    if (bt <= 128) return launch_tc_t<BF16, HAS_LO, 128, 1, 2, 8, 4, 8, 1, 8>(tm, L, p, dev, stream);
    return launch_tc_t<BF16, HAS_LO, 192, 2, 1, 3, 4, 4, 1, 8>(tm, L, p, dev, stream);
  }
  if (pair) {  // per CTA: half of each sub-tile's tokens, so the activation stages are half as large
    if (bt == 256) return launch_tc_t<BF16, HAS_LO, 256, 1, 1, 8, 8, 4, 2>(tm, L, p, dev, stream);
    if (bt == 448) return launch_tc_t<BF16, HAS_LO, 224, 2, 1, 5, 4, 2, 2>(tm, L, p, dev, stream);
    return launch_tc_t<BF16, HAS_LO, 192, 2, 1, 6, 8, 4, 2>(tm, L, p, dev, stream);
  }
  if (bt == 128) return launch_tc_t<BF16, HAS_LO, 128, 1, 2, 8, 8, 8>(tm, L, p, dev, stream);
  if (bt == 256) return launch_tc_t<BF16, HAS_LO, 256, 1, 1, 5, 6, 4>(tm, L, p, dev, stream);
  if (bt == 384) return launch_tc_t<BF16, HAS_LO, 192, 2, 1, 3, 8, 4>(tm, L, p, dev, stream);
  if (bt == 448) return launch_tc_t<BF16, HAS_LO, 224, 2, 1, 3, 4, 2>(tm, L, p, dev, stream);
  return launch_tc_t<BF16, HAS_LO, 192, 1, 2, 6, 8, 4>(tm, L, p, dev, stream);
}

}  // namespace

extern "C" int oc_b200_gptq_gemm_ex(const oc_b200_layer* L, const void* a, int a_dtype, int64_t M, int64_t lda,
                                    const void* bias, int bias_dtype, const void* residual, int64_t ldr, int act,
                                    void* c, int64_t ldc, void* workspace, size_t workspace_bytes,
                                    oc_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (!L) return fail(OC_ERR_INVALID, "gptq_gemm: layer is NULL");
  if (L->kind != 0) return fail(OC_ERR_INVALID, "gptq_gemm: not an AutoGPTQ layer");
  if (M < 0) return fail(OC_ERR_INVALID, "gptq_gemm: M=%lld", (long long)M);
  if (M == 0) return OC_OK;
  if (!a || !c) return fail(OC_ERR_INVALID, "gptq_gemm: NULL activation/output");
  if (!dt16(a_dtype)) return fail(OC_ERR_INVALID, "gptq_gemm: activations must be f16 or bf16");
  if (bias && !dtf(bias_dtype)) return fail(OC_ERR_INVALID, "gptq_gemm: bias dtype");
  if (lda < L->K_in || lda % 8 != 0 || !aligned(a, 16))
    return fail(OC_ERR_INVALID, "gptq_gemm: A must be 16-byte aligned with lda %% 8 == 0 (lda=%lld)", (long long)lda);
  if (ldc < L->N || ldc % 4 != 0 || !aligned(c, 8))
    return fail(OC_ERR_INVALID, "gptq_gemm: C must be 8-byte aligned with ldc %% 4 == 0 (ldc=%lld)", (long long)ldc);
  if (M > 0x7fffffffLL) return fail(OC_ERR_INVALID, "gptq_gemm: M too large");
  if (act != oc::kActNone && act != oc::kActGeluTanh) return fail(OC_ERR_INVALID, "gptq_gemm: act=%d", act);
  if (residual && ldr < L->N) return fail(OC_ERR_INVALID, "gptq_gemm: residual ldr=%lld", (long long)ldr);
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (dev != L->device) return fail(OC_ERR_INVALID, "gptq_gemm: layer lives on device %d, current is %d", L->device, dev);
  const size_t need = oc_b200_gptq_gemm_workspace(L, M);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(OC_ERR_WORKSPACE, "gptq_gemm: workspace needs %zu bytes (got %zu)", need, workspace_bytes);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  unsigned* tickets = reinterpret_cast<unsigned*>(ws);
  size_t off = kTicketBytes;

  if (layer_gemv(L, M) && use_sk(L, M)) {
    float* part = reinterpret_cast<float*>(ws + off);
    return a_dtype == OC_DT_BF16
               ? launch_gemv_sk<true>(L, a, lda, M, bias, bias_dtype, residual, ldr, act, c, ldc, part, tickets, dev,
                                      stream)
               : launch_gemv_sk<false>(L, a, lda, M, bias, bias_dtype, residual, ldr, act, c, ldc, part, tickets, dev,
                                       stream);
  }

  if (layer_gemv(L, M) && use_i8(L, M)) {  // prepares (and gathers) its own activations
    const GemvPlan gp = gemv_plan(L, dev);
    uint8_t* xd = ws + off;
    off += x8_bytes(L, M);
    oc::GemvParams p{};
    p.x = nullptr;
    p.ldx = 0;
    p.M = (int)M;
    p.qw = L->qw;
    p.qz = L->qz;
    p.s = L->s;
    p.s_dtype = L->s_dtype;
    p.wgrp = L->wgrp;
    p.Kp = L->Kp;
    p.N = L->N;
    p.G = L->G;
    p.gs = L->gs;
    p.v1 = L->v1;
    p.bias = bias;
    p.bias_dtype = bias_dtype;
    p.residual = reinterpret_cast<const uint16_t*>(residual);
    p.ldr = ldr;
    p.act = act;
    p.out = reinterpret_cast<uint16_t*>(c);
    p.ldc = ldc;
    p.ws = (gp.splits > 1 && !i8_cluster(gp.splits)) ? reinterpret_cast<float*>(ws + off) : nullptr;
    p.tickets = tickets;
    p.splits = gp.splits;
    p.kstep_per_split = gp.kstep;
    const int n_tiles = (L->N + oc::kGemvCols - 1) / oc::kGemvCols;
    return a_dtype == OC_DT_BF16 ? launch_gemv_i8<true>(L, a, lda, p, gp, n_tiles, xd, stream)
                                 : launch_gemv_i8<false>(L, a, lda, p, gp, n_tiles, xd, stream);
  }

  // activations in kernel K order
  const uint16_t* xk = reinterpret_cast<const uint16_t*>(a);
  int64_t ldx = lda;
  if (L->kperm) {
    uint16_t* xg = reinterpret_cast<uint16_t*>(ws + off);
    off += align_up((size_t)M * L->Kp * 2, 256);
    if (int rc = oc_b200_permute_cols(a, lda, M, L->K_in, L->kperm, L->Kp, xg, stream_)) return rc;
    xk = xg;
    ldx = L->Kp;
  }
  const bool bf16 = a_dtype == OC_DT_BF16;
  const bool has_lo = L->s_dtype != a_dtype;

  if (layer_gemv(L, M)) {
    const GemvPlan gp = gemv_plan(L, dev);
    oc::GemvParams p{};
    p.x = xk;
    p.ldx = ldx;
    p.M = (int)M;
    p.qw = L->qw;
    p.qz = L->qz;
    p.s = L->s;
    p.s_dtype = L->s_dtype;
    p.wgrp = L->wgrp;
    p.Kp = L->Kp;
    p.N = L->N;
    p.G = L->G;
    p.gs = L->gs;
    p.v1 = L->v1;
    p.bias = bias;
    p.bias_dtype = bias_dtype;
    p.residual = reinterpret_cast<const uint16_t*>(residual);
    p.ldr = ldr;
    p.act = act;
    p.out = reinterpret_cast<uint16_t*>(c);
    p.ldc = ldc;
    p.ws = gp.splits > 1 ? reinterpret_cast<float*>(ws + off) : nullptr;
    p.tickets = tickets;
    p.splits = gp.splits;
    p.kstep_per_split = gp.kstep;
    const int n_tiles = (L->N + oc::kGemvCols - 1) / oc::kGemvCols;
    if (legacy_impl(L) == 0)
      return bf16 ? launch_gemv_tcv<true>(L, p, gp, n_tiles, stream) : launch_gemv_tcv<false>(L, p, gp, n_tiles, stream);
    if (legacy_impl(L) == 1)
      return bf16 ? launch_gemv_tma<true>(L, p, gp, n_tiles, stream) : launch_gemv_tma<false>(L, p, gp, n_tiles, stream);
    if (bf16) return has_lo ? launch_gemv<true, true>(p, n_tiles, gp.splits, stream)
                            : launch_gemv<true, false>(p, n_tiles, gp.splits, stream);
    return has_lo ? launch_gemv<false, true>(p, n_tiles, gp.splits, stream)
                  : launch_gemv<false, false>(p, n_tiles, gp.splits, stream);
  }

  int bt = g_opt_tile.load();
  if (bt == 0) bt = choose_tile(M, (L->N + oc::kTcBN - 1) / oc::kTcBN, sm_count(dev));
  if (L->wbits == 8) bt = (bt <= 128) ? 128 : 384;  // the two 8-bit presets
  const CUtensorMapDataType tdt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  TcMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  const bool pair = L->wbits == 4 && use_pairs(M, bt);
  if (pair && bt != 256 && bt != 384 && bt != 448) bt = 384;
  // rows per activation box: tokens per MMA (tiles of 384 / 448 are two sub-tiles), halved for pairs
  const int sub_rows = (bt > 256 ? bt / 2 : bt) / (pair ? 2 : 1);
  if (int rc = make_tmap_2d(&tm.x, tdt, 2, xk, (uint64_t)L->Kp, (uint64_t)M, (uint64_t)ldx * 2, oc::kTcBK,
                            (uint32_t)sub_rows, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  // Output (and residual) tiles go through shared memory by TMA when a tensor map can
  // describe them (16-byte aligned base, row pitch a multiple of 16 bytes); otherwise the
  // epilogue stores directly.
  const bool c_tma = aligned(c, 16) && ldc % 8 == 0;
  const bool r_tma = !residual || (aligned(residual, 16) && ldr % 8 == 0);
  const bool tma_epi = c_tma && r_tma;
  if (tma_epi) {
    if (int rc = make_tmap_2d(&tm.c, tdt, 2, c, (uint64_t)L->N, (uint64_t)M, (uint64_t)ldc * 2, 32, 32,
                              CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
    if (residual)
      if (int rc = make_tmap_2d(&tm.r, tdt, 2, residual, (uint64_t)L->N, (uint64_t)M, (uint64_t)ldr * 2, 32, 32,
                                CU_TENSOR_MAP_SWIZZLE_NONE))
        return rc;
  }
  oc::TcParams p{};
  p.M = (int)M;
  p.N = L->N;
  p.Kp = L->Kp;
  p.qz = L->qz;
  p.s = L->s;
  p.s_dtype = L->s_dtype;
  p.wgrp = L->wgrp;
  p.G = L->G;
  p.gs = L->gs;
  p.v1 = L->v1;
  p.sz_tma = L->sz_tma;
  p.sz_rows = L->sz_rows;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.residual = reinterpret_cast<const uint16_t*>(residual);
  p.ldr = ldr;
  p.act = act;
  p.out = reinterpret_cast<uint16_t*>(c);
  p.ldc = ldc;
  p.tma_epi = tma_epi ? 1 : 0;
  p.n_tiles_n = (L->N + oc::kTcBN * (pair ? 2 : 1) - 1) / (oc::kTcBN * (pair ? 2 : 1));
  p.n_tiles_m = (int)((M + bt - 1) / bt);
  p.num_tiles = p.n_tiles_n * p.n_tiles_m;
  if (bf16) return has_lo ? launch_tc<true, true>(bt, pair, tm, L, p, dev, stream)
                          : launch_tc<true, false>(bt, pair, tm, L, p, dev, stream);
  return has_lo ? launch_tc<false, true>(bt, pair, tm, L, p, dev, stream)
                : launch_tc<false, false>(bt, pair, tm, L, p, dev, stream);
}



// ---------------------------------------------------------------- MoE routing / permutation
extern "C" int oc_b200_moe_route(const void* logits, int logits_dtype, int T, int E, int k, int renorm, int32_t* ids,
                                 float* weights, oc_stream_t stream) {
  if (!logits || !ids || !weights) return fail(OC_ERR_INVALID, "moe_route: NULL pointer");
  if (T < 0 || E <= 0 || E > oc::kMoeMaxE || k <= 0 || k > oc::kMoeMaxK || k > E)
    return fail(OC_ERR_INVALID, "moe_route: T=%d E=%d k=%d", T, E, k);
  if (!dtf(logits_dtype)) return fail(OC_ERR_INVALID, "moe_route: logits dtype");
  if (T == 0) return OC_OK;
  const int threads = 256;
  const int blocks = (T * 32 + threads - 1) / threads;
  oc::moe_route_kernel<<<blocks, threads, 0, stream>>>(logits, logits_dtype, T, E, k, renorm, ids, weights);
  return launch_check("moe_route");
}

extern "C" int oc_b200_moe_permute(const int32_t* ids, int T, int k, int E, int32_t* counts, int32_t* offsets,
                                   int32_t* sorted_token, int32_t* slot_pos, oc_stream_t stream) {
  if (!ids || !counts || !offsets || !sorted_token || !slot_pos) return fail(OC_ERR_INVALID, "moe_permute: NULL");
  if (T < 0 || k <= 0 || E <= 0 || E > oc::kMoeMaxE) return fail(OC_ERR_INVALID, "moe_permute: T=%d k=%d E=%d", T, k, E);
  const int TK = T * k;
  oc::moe_count_kernel<<<E, 256, 0, stream>>>(ids, TK, E, counts);
  oc::moe_scan_kernel<<<1, 256, 0, stream>>>(counts, E, offsets);
  if (TK > 0) oc::moe_scatter_kernel<<<E, 1024, 0, stream>>>(ids, TK, k, offsets, sorted_token, slot_pos);
  return launch_check("moe_permute");
}

extern "C" int oc_b200_gather_rows(const void* src, int64_t lds, const int32_t* idx, int P, int H, void* dst,
                                   int64_t ldd, oc_stream_t stream) {
  if (!src || !idx || !dst) return fail(OC_ERR_INVALID, "gather_rows: NULL pointer");
  if (P < 0 || H <= 0 || H % 8 || lds % 8 || ldd % 8 || !aligned(src, 16) || !aligned(dst, 16))
    return fail(OC_ERR_INVALID, "gather_rows: H=%d must be a multiple of 8 with 16-byte aligned rows", H);
  if (P == 0) return OC_OK;
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  oc::gather_rows_kernel<<<grid_1d((long long)P * (H / 8), 256, dev), 256, 0, stream>>>(
      reinterpret_cast<const uint16_t*>(src), lds, idx, P, H, reinterpret_cast<uint16_t*>(dst), ldd);
  return launch_check("gather_rows");
}

extern "C" int oc_b200_silu_mul(const void* g, const void* u, int64_t ld_in, int P, int F, void* h, int64_t ld_out,
                                int dtype, oc_stream_t stream) {
  if (!g || !u || !h || P < 0 || F <= 0 || !dt16(dtype)) return fail(OC_ERR_INVALID, "silu_mul: bad arguments");
  if (P == 0) return OC_OK;
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  const auto* gg = reinterpret_cast<const uint16_t*>(g);
  const auto* uu = reinterpret_cast<const uint16_t*>(u);
  auto* hh = reinterpret_cast<uint16_t*>(h);
  if (F % 8 == 0 && ld_in % 8 == 0 && ld_out % 8 == 0 && aligned(g, 16) && aligned(u, 16) && aligned(h, 16)) {
    const int blocks = grid_1d((long long)P * (F / 8), 256, dev);
    if (dtype == OC_DT_BF16)
      oc::silu_mul_v8_kernel<true><<<blocks, 256, 0, stream>>>(gg, uu, ld_in, P, F / 8, hh, ld_out);
    else
      oc::silu_mul_v8_kernel<false><<<blocks, 256, 0, stream>>>(gg, uu, ld_in, P, F / 8, hh, ld_out);
    return launch_check("silu_mul");
  }
  const int blocks = grid_1d((long long)P * F, 256, dev);
  if (dtype == OC_DT_BF16)
    oc::silu_mul_kernel<true><<<blocks, 256, 0, stream>>>(gg, uu, ld_in, P, F, hh, ld_out);
  else
    oc::silu_mul_kernel<false><<<blocks, 256, 0, stream>>>(gg, uu, ld_in, P, F, hh, ld_out);
  return launch_check("silu_mul");
}

extern "C" int oc_b200_moe_combine(const void* y, int64_t ldy, const int32_t* slot_pos, const float* w, int T, int k,
                                   int H, const void* shared, int64_t lds, void* out, int64_t ldo, int dtype,
                                   oc_stream_t stream) {
  if (!y || !slot_pos || !w || !out || T < 0 || k <= 0 || H <= 0 || !dt16(dtype))
    return fail(OC_ERR_INVALID, "moe_combine: bad arguments");
  if (T == 0) return OC_OK;
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  const auto* yy = reinterpret_cast<const uint16_t*>(y);
  const auto* sh = reinterpret_cast<const uint16_t*>(shared);
  auto* o = reinterpret_cast<uint16_t*>(out);
  if (H % 8 == 0 && ldy % 8 == 0 && ldo % 8 == 0 && aligned(y, 16) && aligned(out, 16) &&
      (!shared || (lds % 8 == 0 && aligned(shared, 16)))) {
    const int blocks = grid_1d((long long)T * (H / 8), 256, dev);
    if (dtype == OC_DT_BF16)
      oc::moe_combine_v8_kernel<true><<<blocks, 256, 0, stream>>>(yy, ldy, slot_pos, w, T, k, H / 8, sh, lds, o, ldo);
    else
      oc::moe_combine_v8_kernel<false><<<blocks, 256, 0, stream>>>(yy, ldy, slot_pos, w, T, k, H / 8, sh, lds, o, ldo);
    return launch_check("moe_combine");
  }
  const int blocks = grid_1d((long long)T * H, 256, dev);
  if (dtype == OC_DT_BF16)
    oc::moe_combine_kernel<true><<<blocks, 256, 0, stream>>>(yy, ldy, slot_pos, w, T, k, H, sh, lds, o, ldo);
  else
    oc::moe_combine_kernel<false><<<blocks, 256, 0, stream>>>(yy, ldy, slot_pos, w, T, k, H, sh, lds, o, ldo);
  return launch_check("moe_combine");
}

// ---------------------------------------------------------------- row-packed (RTN / DSV4) layers
namespace {
// [E weight maps][E scale maps][E zero maps] then [E scale pointers][E zero pointers]
size_t rows_maps_bytes(int E) { return align_up((size_t)3 * E * sizeof(CUtensorMap), 256); }
size_t rows_table_bytes(int E) { return rows_maps_bytes(E) + align_up((size_t)E * 16, 256); }
}

extern "C" size_t oc_b200_rows_table_bytes(int E) { return E > 0 ? rows_table_bytes(E) : 0; }

extern "C" int oc_b200_rows_layer_create(int E, const uint8_t* const* packed, int64_t ld_bytes, int wbits,
                                         const void* const* scales, int scales_dtype, const void* const* zeros,
                                         int zeros_dtype, int64_t stride_n, int64_t stride_g, int groupsize, int K,
                                         int N, int mode, void* table, oc_stream_t stream_, oc_b200_layer** out) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (!out) return fail(OC_ERR_INVALID, "rows_layer_create: out is NULL");
  *out = nullptr;
  if (E <= 0 || E > oc::kRowsMaxE) return fail(OC_ERR_INVALID, "rows_layer_create: E=%d (1..%d)", E, oc::kRowsMaxE);
  if (!packed || !scales || !zeros || !table) return fail(OC_ERR_INVALID, "rows_layer_create: NULL pointer");
  if (wbits != 2 && wbits != 4) return fail(OC_ERR_UNSUPPORTED, "rows_layer_create: wbits=%d", wbits);
  if (mode != 0 && mode != 1) return fail(OC_ERR_INVALID, "rows_layer_create: mode=%d", mode);
  if (mode == 1 && wbits != 4) return fail(OC_ERR_UNSUPPORTED, "rows_layer_create: RTN layers are 4-bit");
  const int span = 32 / wbits;
  if (K <= 0 || N <= 0 || K % 8 != 0) return fail(OC_ERR_INVALID, "rows_layer_create: K=%d N=%d", K, N);
  if (ld_bytes * (8 / wbits) < K || ld_bytes % 16 != 0)
    return fail(OC_ERR_UNSUPPORTED, "rows_layer_create: row stride %lld bytes must cover K and be a multiple of 16",
                (long long)ld_bytes);
  if (groupsize <= 0 || (groupsize % span != 0 && groupsize < K))
    return fail(OC_ERR_UNSUPPORTED, "rows_layer_create: groupsize %d must be a multiple of %d", groupsize, span);
  if (!dtf(scales_dtype) || !dtf(zeros_dtype)) return fail(OC_ERR_INVALID, "rows_layer_create: dtype");
  if (!aligned(table, 256)) return fail(OC_ERR_INVALID, "rows_layer_create: table must be 256-byte aligned");
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (int rc = oc_b200_device_check(dev)) return rc;
  const size_t maps_bytes = rows_maps_bytes(E);
  uint8_t* host = new uint8_t[rows_table_bytes(E)]();
  CUtensorMap* maps = reinterpret_cast<CUtensorMap*>(host);
  CUtensorMap* smaps = maps + E;
  CUtensorMap* zmaps = maps + 2 * E;
  const void** sp = reinterpret_cast<const void**>(host + maps_bytes);
  const void** zp = sp + E;
  // Scales / zeros stored [G, N] (stride_n == 1) ride in each weight stage by TMA: the rows of the
  // groups one 64-k block covers, 128 features each, when they fit the stage's 512 bytes per tensor.
  const int span_k = 32 / wbits;
  const int gs_eff = groupsize >= K ? (K + span_k - 1) / span_k * span_k : groupsize;
  const int G = (K + gs_eff - 1) / gs_eff;
  const int sz_rows = (gs_eff < 64 && 64 % gs_eff == 0) ? 64 / gs_eff : 1;
  const int s_es = scales_dtype == OC_DT_F32 ? 4 : 2, z_es = zeros_dtype == OC_DT_F32 ? 4 : 2;
  bool sz_tma = stride_n == 1 && stride_g >= N && (G == 1 || gs_eff % 64 == 0 || 64 % gs_eff == 0) &&
                sz_rows * 128 * s_es <= 512 && sz_rows * 128 * z_es <= 512 && (stride_g * s_es) % 16 == 0 &&
                (stride_g * z_es) % 16 == 0;
  for (int e = 0; e < E; ++e) {
    if (!packed[e] || !scales[e] || !zeros[e]) {
      delete[] host;
      return fail(OC_ERR_INVALID, "rows_layer_create: NULL tensor for expert %d", e);
    }
    if (int rc = make_tmap_2d(&maps[e], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, packed[e], (uint64_t)ld_bytes, (uint64_t)N,
                              (uint64_t)ld_bytes, (uint32_t)(64 * wbits / 8), 128, CU_TENSOR_MAP_SWIZZLE_NONE)) {
      delete[] host;
      return rc;
    }
    sp[e] = scales[e];
    zp[e] = zeros[e];
    if (sz_tma && (!aligned(scales[e], 16) || !aligned(zeros[e], 16))) sz_tma = false;
  }
  if (sz_tma) {
    const auto sdt = s_es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const auto zdt = z_es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    for (int e = 0; e < E && sz_tma; ++e) {
      if (make_tmap_2d(&smaps[e], sdt, s_es, scales[e], (uint64_t)N, (uint64_t)G, (uint64_t)stride_g * s_es, 128,
                       (uint32_t)sz_rows, CU_TENSOR_MAP_SWIZZLE_NONE) != OC_OK ||
          make_tmap_2d(&zmaps[e], zdt, z_es, zeros[e], (uint64_t)N, (uint64_t)G, (uint64_t)stride_g * z_es, 128,
                       (uint32_t)sz_rows, CU_TENSOR_MAP_SWIZZLE_NONE) != OC_OK)
        sz_tma = false;
    }
    g_last_error.clear();
  }
  int rc = cuda_check(cudaMemcpyAsync(table, host, rows_table_bytes(E), cudaMemcpyHostToDevice, stream), "table copy");
  if (!rc) rc = cuda_check(cudaStreamSynchronize(stream), "table copy sync");
  delete[] host;
  if (rc) return rc;
  auto* L = new oc_b200_layer();
  L->kind = 1;
  L->device = dev;
  L->E = E;
  L->wbits = wbits;
  L->mode = mode;
  L->s_dtype_r = scales_dtype;
  L->z_dtype_r = zeros_dtype;
  L->stride_n = stride_n;
  L->stride_g = stride_g;
  // one group per row when groupsize covers K (any K % span is then harmless)
  L->gs = groupsize >= K ? (K + span - 1) / span * span : groupsize;
  L->K_in = K;
  L->Kp = K;
  L->N = N;
  L->d_wmaps = reinterpret_cast<const CUtensorMap*>(table);
  L->d_sptr = reinterpret_cast<const void* const*>(reinterpret_cast<uint8_t*>(table) + maps_bytes);
  L->d_zptr = L->d_sptr + E;
  L->sz_tma = sz_tma ? 1 : 0;
  L->sz_rows = sz_rows;
  *out = L;
  return OC_OK;
}

namespace {

template <bool BF16, int WB, int MODE, bool HL, int BT, int ACC, int XS, int WS, int AS, bool SWIGLU = false>
int launch_rows_t(const CUtensorMap& tx, const oc::RowsParams& p, int dev, cudaStream_t stream) {
  using Cfg = oc::RowsCfg<WB, BT, ACC, XS, WS, AS, SWIGLU>;
  auto kern = oc::rows_gemm_tc_kernel<BF16, WB, MODE, HL, BT, ACC, XS, WS, AS, SWIGLU>;
  static bool attr_set[kMaxDevices] = {};
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes),
                            "cudaFuncSetAttribute(smem)"))
      return rc;
    attr_set[dev] = true;
  }
  // upper bound on tiles: every expert segment adds at most one partial m-tile
  const long long m_tiles = ((long long)p.M + BT - 1) / BT + (p.offsets ? p.E : 0);
  const long long tiles = m_tiles * p.n_tiles_n;
  const int grid = tiles < tc_ctas(dev) ? (int)tiles : tc_ctas(dev);
  kern<<<grid, oc::kRowsThreads, Cfg::kSmemBytes, stream>>>(tx, p);
  return launch_check("rows_gemm_tc");
}

template <bool BF16, int WB, int MODE, bool HL>
int launch_rows_bt(int bt, const CUtensorMap& tx, const oc::RowsParams& p, int dev, cudaStream_t stream,
                   bool swiglu) {
  // The weight ring is deep (16-32 stages of 3-5 KB) because packed weights stream from HBM with
  // ~2 us of latency; activation tiles come from L2 and need fewer stages.
  if (swiglu) {
    // A tile takes both slots of a two-slot accumulator ring (gate, up). Measured alternatives at
    // config 3's routed experts, all slower than this (2.77 ms): 80-token tiles with three slots
    // beside 8 A stages (epilogue overlapped; 2.84 ms), three 128-token slots beside 4 A stages,
    // or the gate outputs parked in shared memory (2.83-2.86 ms). Dense: 192-token tiles.
    if (bt == 128) {
      if constexpr (WB == 2)
        return launch_rows_t<BF16, WB, MODE, HL, 128, 2, 6, 32, 8, true>(tx, p, dev, stream);
      else
        return launch_rows_t<BF16, WB, MODE, HL, 128, 2, 4, 24, 8, true>(tx, p, dev, stream);
    }
    return launch_rows_t<BF16, WB, MODE, HL, 192, 2, 5, 16, 4, true>(tx, p, dev, stream);
  }
  if (bt == 128) {
    if constexpr (WB == 2)
      return launch_rows_t<BF16, WB, MODE, HL, 128, 2, 6, 32, 8>(tx, p, dev, stream);
    else
      return launch_rows_t<BF16, WB, MODE, HL, 128, 2, 4, 24, 8>(tx, p, dev, stream);
  }
  return launch_rows_t<BF16, WB, MODE, HL, 192, 2, 5, 16, 4>(tx, p, dev, stream);
}

template <bool BF16>
int launch_rows(int bt, int wbits, int mode, bool has_lo, const CUtensorMap& tx, const oc::RowsParams& p, int dev,
                cudaStream_t stream, bool swiglu) {
  if (mode == oc::kRowsRtn) return launch_rows_bt<BF16, 4, oc::kRowsRtn, false>(bt, tx, p, dev, stream, swiglu);
  if (wbits == 4)
    return has_lo ? launch_rows_bt<BF16, 4, oc::kRowsExact, true>(bt, tx, p, dev, stream, swiglu)
                  : launch_rows_bt<BF16, 4, oc::kRowsExact, false>(bt, tx, p, dev, stream, swiglu);
  return has_lo ? launch_rows_bt<BF16, 2, oc::kRowsExact, true>(bt, tx, p, dev, stream, swiglu)
                : launch_rows_bt<BF16, 2, oc::kRowsExact, false>(bt, tx, p, dev, stream, swiglu);
}

// Shared body of oc_b200_rows_gemm and oc_b200_rows_gemm_swiglu (swiglu: the layer is the [F, 2K]
// gate|up matrix; A has K = K_in / 2 columns and C gets silu(gate) * up, F columns).
int rows_gemm_impl(const oc_b200_layer* L, const void* a, int a_dtype, int64_t M, int64_t lda, const int32_t* offsets,
                   const void* bias, int bias_dtype, void* c, int64_t ldc, cudaStream_t stream, bool swiglu) {
  const char* nm = swiglu ? "rows_gemm_swiglu" : "rows_gemm";
  if (!L || L->kind != 1) return fail(OC_ERR_INVALID, "%s: not a row-packed layer", nm);
  if (M < 0) return fail(OC_ERR_INVALID, "%s: M=%lld", nm, (long long)M);
  const int k_act = swiglu ? L->K_in / 2 : L->K_in;
  if (swiglu && (L->K_in % 128 != 0 || L->gs >= L->K_in || k_act % L->gs != 0))
    return fail(OC_ERR_INVALID,
                "%s: the layer must be a gate|up matrix of 2K columns with K a multiple of 64 and of the groupsize "
                "(K_in=%d, groupsize=%d)", nm, L->K_in, L->gs);
  if (M == 0) return OC_OK;
  if (!a || !c) return fail(OC_ERR_INVALID, "%s: NULL activation/output", nm);
  if (!dt16(a_dtype)) return fail(OC_ERR_INVALID, "%s: activations must be f16 or bf16", nm);
  if (L->E > 1 && !offsets) return fail(OC_ERR_INVALID, "%s: expert groups need offsets", nm);
  if (bias && (offsets || swiglu || !dtf(bias_dtype))) return fail(OC_ERR_INVALID, "%s: bias (dense layers only)", nm);
  if (lda < k_act || lda % 8 != 0 || !aligned(a, 16))
    return fail(OC_ERR_INVALID, "%s: A must be 16-byte aligned with lda %% 8 == 0", nm);
  if (ldc < L->N || !aligned(c, 2)) return fail(OC_ERR_INVALID, "%s: ldc", nm);
  if (M > 0x7fffffffLL) return fail(OC_ERR_INVALID, "%s: M too large", nm);
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (dev != L->device) return fail(OC_ERR_INVALID, "%s: layer lives on device %d", nm, L->device);
  const bool bf16 = a_dtype == OC_DT_BF16;
  int bt = g_opt_tile.load();
  if (bt != 128 && bt != 192) bt = offsets ? 128 : 192;
  CUtensorMap tx;
  if (int rc = make_tmap_2d(&tx, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a,
                            (uint64_t)k_act, (uint64_t)M, (uint64_t)lda * 2, 64, (uint32_t)bt,
                            CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  oc::RowsParams p{};
  p.M = (int)M;
  p.N = L->N;
  p.K = L->K_in;
  p.kb_x = k_act / 64;
  p.E = L->E;
  p.offsets = offsets;
  p.wmaps = L->d_wmaps;
  p.smaps = L->d_wmaps + L->E;
  p.zmaps = L->d_wmaps + 2 * L->E;
  p.sptr = L->d_sptr;
  p.zptr = L->d_zptr;
  p.sz_tma = L->sz_tma;
  p.sz_rows = L->sz_rows;
  p.s_es = L->s_dtype_r == OC_DT_F32 ? 4 : 2;
  p.z_es = L->z_dtype_r == OC_DT_F32 ? 4 : 2;
  p.s_dtype = L->s_dtype_r;
  p.z_dtype = L->z_dtype_r;
  p.s_stride_n = L->stride_n;
  p.s_stride_g = L->stride_g;
  p.gs = L->gs;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.out = reinterpret_cast<uint16_t*>(c);
  p.ldc = ldc;
  p.n_tiles_n = (L->N + 127) / 128;
  const bool has_lo = L->s_dtype_r != a_dtype;
  if (bf16) return launch_rows<true>(bt, L->wbits, L->mode, has_lo, tx, p, dev, stream, swiglu);
  return launch_rows<false>(bt, L->wbits, L->mode, has_lo, tx, p, dev, stream, swiglu);
}

}  // namespace

extern "C" int oc_b200_rows_gemm(const oc_b200_layer* L, const void* a, int a_dtype, int64_t M, int64_t lda,
                                 const int32_t* offsets, const void* bias, int bias_dtype, void* c, int64_t ldc,
                                 oc_stream_t stream) {
  return rows_gemm_impl(L, a, a_dtype, M, lda, offsets, bias, bias_dtype, c, ldc,
                        reinterpret_cast<cudaStream_t>(stream), false);
}

extern "C" int oc_b200_rows_gemm_swiglu(const oc_b200_layer* L, const void* a, int a_dtype, int64_t M, int64_t lda,
                                        const int32_t* offsets, void* c, int64_t ldc, oc_stream_t stream) {
  return rows_gemm_impl(L, a, a_dtype, M, lda, offsets, nullptr, 0, c, ldc, reinterpret_cast<cudaStream_t>(stream),
                        true);
}

// ---------------------------------------------------------------- decode GEMV without a workspace
// For callers that cannot allocate device memory when they call (see oc_b200_gptq_gemv_noalloc
// in the header): the split-K partials, the act-order gather and the column tickets live in
// this fixed array instead of a caller workspace. The tickets (first kTicketBytes) must be
// zero before the first launch; the one-time setup zeroes them and every launch leaves them
// zero again. One array per device (a __device__ variable exists once per device context),
// so concurrent calls on one device race on it.
namespace {
constexpr size_t kNoAllocScratchBytes = OC_B200_NOALLOC_SCRATCH_BYTES;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
std::atomic<void*> g_noalloc_ptr[kMaxDevices];

// Address of this device's scratch (the device must be current); the first call per device
// looks it up, zeroes the tickets and waits for the device, so it belongs before any capture.
int noalloc_scratch(int dev, uint8_t** out) {
  if (dev < 0 || dev >= kMaxDevices) return fail(OC_ERR_INVALID, "gemv_noalloc: device %d out of range", dev);
  void* ptr = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (!ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    ptr = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
    if (!ptr) {
      if (int rc = cuda_check(cudaGetSymbolAddress(&ptr, g_noalloc_scratch), "cudaGetSymbolAddress(noalloc scratch)"))
        return rc;
      if (int rc = cuda_check(cudaMemset(ptr, 0, kTicketBytes), "cudaMemset(noalloc tickets)")) return rc;
      if (int rc = cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize(noalloc setup)")) return rc;
      g_noalloc_ptr[dev].store(ptr, std::memory_order_release);
    }
  }
  *out = reinterpret_cast<uint8_t*>(ptr);
  return OC_OK;
}
}  // namespace

extern "C" int oc_b200_gptq_gemv_noalloc(const oc_b200_layer* L, const void* a, int a_dtype, int64_t M, int64_t lda,
                                         const void* bias, int bias_dtype, void* c, int64_t ldc,
                                         oc_stream_t stream_) {
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (!L) return fail(OC_ERR_INVALID, "gemv_noalloc: layer is NULL");
  if (L->kind != 0) return fail(OC_ERR_INVALID, "gemv_noalloc: not an AutoGPTQ layer");
  if (M < 0 || M > 16) return fail(OC_ERR_INVALID, "gemv_noalloc: M=%lld (takes 0 <= M <= 16)", (long long)M);
  if (M == 0) return OC_OK;
  if (!a || !c) return fail(OC_ERR_INVALID, "gemv_noalloc: NULL activation/output");
  if (!dt16(a_dtype)) return fail(OC_ERR_INVALID, "gemv_noalloc: activations must be f16 or bf16");
  if (bias && !dtf(bias_dtype)) return fail(OC_ERR_INVALID, "gemv_noalloc: bias dtype");
  if (lda < L->K_in || lda % 8 != 0 || !aligned(a, 16))
    return fail(OC_ERR_INVALID, "gemv_noalloc: A must be 16-byte aligned with lda %% 8 == 0 (lda=%lld)",
                (long long)lda);
  if (ldc < L->N || ldc % 4 != 0 || !aligned(c, 8))
    return fail(OC_ERR_INVALID, "gemv_noalloc: C must be 8-byte aligned with ldc %% 4 == 0 (ldc=%lld)",
                (long long)ldc);
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  if (dev != L->device)
    return fail(OC_ERR_INVALID, "gemv_noalloc: layer lives on device %d, current is %d", L->device, dev);
  const GemvPlan gp = gemv_plan(L, dev);
  size_t need = kTicketBytes;
  const size_t gather_bytes = L->kperm ? align_up((size_t)M * L->Kp * 2, 256) : 0;
  need += gather_bytes;
  if (gp.splits > 1) need += align_up((size_t)gp.splits * M * L->N * 4, 256);
  if (need > kNoAllocScratchBytes)
    return fail(OC_ERR_INVALID, "gemv_noalloc: needs %zu bytes of scratch, the fixed scratch holds %zu (M=%lld N=%d)",
                need, kNoAllocScratchBytes, (long long)M, L->N);
  uint8_t* ws = nullptr;
  if (int rc = noalloc_scratch(dev, &ws)) return rc;
  unsigned* tickets = reinterpret_cast<unsigned*>(ws);
  size_t off = kTicketBytes;
  const uint16_t* xk = reinterpret_cast<const uint16_t*>(a);
  int64_t ldx = lda;
  if (L->kperm) {
    uint16_t* xg = reinterpret_cast<uint16_t*>(ws + off);
    off += gather_bytes;
    if (int rc = oc_b200_permute_cols(a, lda, M, L->K_in, L->kperm, L->Kp, xg, stream_)) return rc;
    xk = xg;
    ldx = L->Kp;
  }
  oc::GemvParams p{};
  p.x = xk;
  p.ldx = ldx;
  p.M = (int)M;
  p.qw = L->qw;
  p.qz = L->qz;
  p.s = L->s;
  p.s_dtype = L->s_dtype;
  p.wgrp = L->wgrp;
  p.Kp = L->Kp;
  p.N = L->N;
  p.G = L->G;
  p.gs = L->gs;
  p.v1 = L->v1;
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.residual = nullptr;
  p.ldr = 0;
  p.act = oc::kActNone;
  p.out = reinterpret_cast<uint16_t*>(c);
  p.ldc = ldc;
  p.ws = gp.splits > 1 ? reinterpret_cast<float*>(ws + off) : nullptr;
  p.tickets = tickets;
  p.splits = gp.splits;
  p.kstep_per_split = gp.kstep;
  const int n_tiles = (L->N + oc::kGemvCols - 1) / oc::kGemvCols;
  const bool bf16 = a_dtype == OC_DT_BF16;
  const bool has_lo = L->s_dtype != a_dtype;
  if (legacy_impl(L) == 0)
    return bf16 ? launch_gemv_tcv<true>(L, p, gp, n_tiles, stream) : launch_gemv_tcv<false>(L, p, gp, n_tiles, stream);
  if (legacy_impl(L) == 1)
    return bf16 ? launch_gemv_tma<true>(L, p, gp, n_tiles, stream) : launch_gemv_tma<false>(L, p, gp, n_tiles, stream);
  if (bf16) return has_lo ? launch_gemv<true, true>(p, n_tiles, gp.splits, stream)
                          : launch_gemv<true, false>(p, n_tiles, gp.splits, stream);
  return has_lo ? launch_gemv<false, true>(p, n_tiles, gp.splits, stream)
                : launch_gemv<false, false>(p, n_tiles, gp.splits, stream);
}

extern "C" int oc_b200_gptq_gemm(const oc_b200_layer* L, const void* a, int a_dtype, int64_t M, int64_t lda,
                                 const void* bias, int bias_dtype, void* c, int64_t ldc, void* workspace,
                                 size_t workspace_bytes, oc_stream_t stream) {
  return oc_b200_gptq_gemm_ex(L, a, a_dtype, M, lda, bias, bias_dtype, nullptr, 0, oc::kActNone, c, ldc, workspace,
                              workspace_bytes, stream);
}
