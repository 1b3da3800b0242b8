// Shared device helpers for the onecomp B200 kernels (sm_100a only).
//
// * dtype tags and scalar load/convert helpers;
// * packed bf16x2 / f16x2 arithmetic written as explicit PTX so every
//   rounding is the IEEE round-to-nearest-even of the exact result;
// * mbarrier / TMA / tcgen05 wrappers;
// * bounded waits: every spin has an iteration limit after which the kernel
//   records an error code in `g_oc_dev_error` and the caller unwinds.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef OC_WAIT_NS
// Wall-clock bound of every spin-wait (device %globaltimer, ns): far above any
// legitimate wait (a whole tile takes well under a millisecond), far below a hang.
#define OC_WAIT_NS 2000000000ull
#endif

namespace oc {

enum DType : int { kF16 = 0, kBF16 = 1, kF32 = 2 };

// Device-side error word. 0 = ok; otherwise a code identifying the wait that
// gave up (see OC_DEVERR_*). Read and cleared by oc_b200_read_device_error().
__device__ unsigned int g_oc_dev_error;

enum : unsigned {
  kDevErrTmaFull = 0x101,
  kDevErrTmaEmpty = 0x102,
  kDevErrAFull = 0x103,
  kDevErrAEmpty = 0x104,
  kDevErrAccFull = 0x105,
  kDevErrAccEmpty = 0x106,
  kDevErrWFull = 0x107,
  kDevErrWEmpty = 0x108,
  kDevErrDrain = 0x109,
  kDevErrResFull = 0x10a,
  kDevErrIndex = 0x301,   // embedding id outside the table
  kDevErrSplitK = 0x201,
  kDevErrCluster = 0x202,  // a cluster split-K reduction gave up waiting for a CTA of its cluster
};

__device__ __forceinline__ void record_error(unsigned code) { atomicCAS(&g_oc_dev_error, 0u, code); }

// ----------------------------------------------------------------------------
// scalar conversions
// ----------------------------------------------------------------------------
__device__ __forceinline__ float load_as_f32(const void* p, int dtype, long long i) {
  if (dtype == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dtype == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ uint16_t f32_to_bits(float v, int dtype) {
  if (dtype == kF16) return __half_as_ushort(__float2half_rn(v));
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float bits_to_f32(uint16_t b, int dtype) {
  if (dtype == kF16) return __half2float(__ushort_as_half(b));
  return __bfloat162float(__ushort_as_bfloat16(b));
}

// GEMM epilogue activations
enum Act : int { kActNone = 0, kActGeluTanh = 1 };

// tanh-approximated GELU, 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))), the formula of
// torch.nn.functional.gelu(approximate="tanh"); tanh from the hardware approximation
// (tanh.approx.f32, relative error ~2^-11, below the 2^-8 spacing of the 16-bit output).
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// silu(g) = g / (1 + e^-g) with the fast exponential and division intrinsics (a few fp32 ulps
// from the exact value, far below the 16-bit rounding that follows): the MoE expert activation,
// shared by the silu-mul kernel and the fused gate|up GEMM epilogue so both give the same bits.
// Large negative g: e^-g overflows to inf, the fast division gives (-)0, the limit of silu.
__device__ __forceinline__ float silu_f32(float g) { return __fdividef(g, 1.f + __expf(-g)); }

__device__ __forceinline__ float gelu_tanh(float v) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * v, v * v, v);
  const float h = 0.5f * v;
  return fmaf(h, tanh_approx(u), h);
}

__device__ __forceinline__ float epilogue_value(float acc, float bias, int act, const uint16_t* residual,
                                                int dtype) {
  float v = acc + bias;
  if (act == kActGeluTanh) v = gelu_tanh(v);
  if (residual) v += bits_to_f32(*residual, dtype);
  return v;
}

// ----------------------------------------------------------------------------
// packed 16-bit pair arithmetic (each op rounds the exact result once, RNE)
// ----------------------------------------------------------------------------
template <bool BF16> struct Pair;

template <> struct Pair<true> {
  // 128.0 in bf16: OR-ing a 4-bit code into the low mantissa bits gives 128 + q exactly.
  static constexpr uint32_t kMagic = 0x43004300u;
  static constexpr float kMagicF = 128.0f;
  __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t d; asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b)); return d;
  }
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d; asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b)); return d;
  }
  __device__ __forceinline__ static uint32_t fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d; asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
  }
  __device__ __forceinline__ static uint16_t from_f32(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }
  __device__ __forceinline__ static float to_f32(uint16_t b) { return __bfloat162float(__ushort_as_bfloat16(b)); }
};

template <> struct Pair<false> {
  // 1024.0 in fp16: 1024 + q exactly for a 4-bit code.
  static constexpr uint32_t kMagic = 0x64006400u;
  static constexpr float kMagicF = 1024.0f;
  __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t d; asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b)); return d;
  }
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d; asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b)); return d;
  }
  __device__ __forceinline__ static uint32_t fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d; asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
  }
  __device__ __forceinline__ static uint16_t from_f32(float v) { return __half_as_ushort(__float2half_rn(v)); }
  __device__ __forceinline__ static float to_f32(uint16_t b) { return __half2float(__ushort_as_half(b)); }
};

// Two fp32 values rounded (to nearest even) to a bf16x2 / f16x2 pair: lo in the low half.
template <bool BF16>
__device__ __forceinline__ uint32_t pack2_rn(float lo, float hi) {
  if constexpr (BF16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(magic));  // (a & b) | c
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d; asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel)); return d;
}

__device__ __forceinline__ uint32_t pack2(uint16_t lo, uint16_t hi) { return (uint32_t)lo | ((uint32_t)hi << 16); }

// Per-(group, row) dequant constants for the exact packed path.
//   w = RNE( s * (q - z) ) computed as  d = (M+q) - (M+z)            (exact)
//                                       w = fma(d, s_hi, d * s_lo)   (one rounding)
// with s_hi = RNE(s) in the pair type and s_lo = s - s_hi (exact, <= 3 bits),
// so d * s_lo is exact and the fma rounds d*s exactly once.
template <bool BF16> struct DqConst {
  uint32_t zm;   // (M+z, M+z)
  uint32_t shi;  // (s_hi, s_hi)
  uint32_t slo;  // (s_lo, s_lo)
};

template <bool BF16>
__device__ __forceinline__ DqConst<BF16> make_dq_const(float s, int z) {
  using P = Pair<BF16>;
  DqConst<BF16> c;
  const uint16_t zm = P::from_f32(P::kMagicF + (float)z);
  const uint16_t hi = P::from_f32(s);
  const uint16_t lo = P::from_f32(s - P::to_f32(hi));
  c.zm = pack2(zm, zm);
  c.shi = pack2(hi, hi);
  c.slo = pack2(lo, lo);
  return c;
}

// Is the split s = s_hi + s_lo of make_dq_const exact and its products exact, so that
// fma(d, s_hi, d * s_lo) rounds d * s once for every d with at most 5 significant bits?
//   * s_hi must be finite and s_hi + s_lo == s (an fp32 sum that is exact whenever the split is);
//   * s_lo = 0, or (bf16 pairs) s_lo has at most 3 significant bits (d * s_lo then fits the 8-bit
//     pair mantissa) and is far above bf16's underflow. fp16 pairs need s_lo = 0: a nonzero s_lo
//     times d may fall below fp16's subnormal range.
// Always true for positive fp16 scales with bf16 pairs and for positive scales of the pair's
// own dtype.
template <bool BF16>
__device__ __forceinline__ bool split_exact(float s, uint16_t hi, uint16_t lo) {
  using P = Pair<BF16>;
  const float hf = P::to_f32(hi), lf = P::to_f32(lo);
  if (!(s > 0.f) || !isfinite(hf) || hf + lf != s) return false;  // (signed zeros of s <= 0 differ)
  if (lf == 0.f) return true;
  if (!BF16) return false;
  return (__float_as_uint(lf) & 0x1FFFFFu) == 0u && fabsf(lf) >= 0x1p-110f;
}

template <bool BF16>
__device__ __forceinline__ bool dq_const_exact(float s, const DqConst<BF16>& c) {
  return split_exact<BF16>(s, (uint16_t)(c.shi & 0xFFFFu), (uint16_t)(c.slo & 0xFFFFu));
}

template <bool BF16, bool HAS_LO>
__device__ __forceinline__ uint32_t dq_pair(uint32_t magic_q, const DqConst<BF16>& c) {
  using P = Pair<BF16>;
  const uint32_t d = P::sub(magic_q, c.zm);
  if (HAS_LO) return P::fma(d, c.shi, P::mul(d, c.slo));
  return P::mul(d, c.shi);
}

// ----------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: returns false (and records `code`) if the phase does not complete
// within `limit_ns`, or as soon as another role of this CTA has aborted.
__device__ __forceinline__ bool mbar_wait_ns(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                             unsigned code, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 0u) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > limit_ns) break;
    }
  }
  record_error(code);
  *abort_flag = 1;
  return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned code) {
  return mbar_wait_ns(bar, parity, abort_flag, code, OC_WAIT_NS);
}

// Bounded wait used while unwinding after an abort (no abort-flag check).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > OC_WAIT_NS) {
      record_error(kDevErrDrain);
      return;
    }
  }
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------------
// TMA (no multicast anywhere in this code base)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Tiled TMA store smem -> global (bulk-group completion). Coordinates are non-negative;
// parts of the box outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until all but the N most recent committed bulk-store groups have finished reading
// their shared-memory source.
template <int N> __device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Named barrier over `count` threads (a multiple of 32) of the CTA.
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Named barrier that also ORs a predicate over the participating threads.
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// L2 prefetch of one tiled box (no shared memory, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
// L2 prefetch of a contiguous range (16-byte aligned address, size a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------------------------
// tcgen05 (cta_group::1 only)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- CTA pairs (cluster of 2, tcgen05 cta_group::2) ----------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster (shared::cluster window).
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Arrive (release, cluster scope) on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Bounded wait on a local mbarrier whose arrivals come from other CTAs of the cluster (acquire at
// cluster scope, so their shared-memory writes before the arrival are visible). Records `code`
// and returns false when the phase does not complete within `limit_ns`.
__device__ __forceinline__ bool mbar_wait_cluster_ns(uint64_t* bar, uint32_t parity, unsigned code,
                                                     uint64_t limit_ns) {
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 15u) == 15u && global_timer_ns() - t0 > limit_ns) break;
  }
  record_error(code);
  return false;
}
// Loads from another CTA's shared memory (a shared::cluster address from mapa_shared).
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ int ld_dsmem_s32(uint32_t addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void tmem_alloc_cg2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_cg2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_cg2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrive on the barrier at the same offset in every CTA of `mask` once all prior MMAs of the
// pair (issued by this thread) have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                   "r"(smem_u32(bar)),
               "h"(mask)
               : "memory");
}
// D[tmem] (+)= A[tmem] x B[smem desc] over the CTA pair: M = 256 (128 rows of A and D in each
// CTA's TMEM), B split by N between the two CTAs' shared memory at the same offset.
__device__ __forceinline__ void tc_mma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Tiled TMA load of a CTA pair: the completion is signalled on an mbarrier given by its
// shared::cluster address, which may sit in the peer CTA (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// D[tmem] (+)= A[tmem] x B[smem desc]
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit: thread i of the warp owns lane (base lane + i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

// K-major operand in shared memory with the 128-byte swizzle: rows of 64 16-bit
// elements (128 B), 8-row atoms 1024 B apart. `addr` must sit in a 1024-B aligned tile.
__device__ __forceinline__ uint64_t smem_desc_kmajor_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);        // start address
  d |= (uint64_t)1 << 16;                          // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;               // stride byte offset between 8-row atoms
  d |= (uint64_t)1 << 46;                          // descriptor version (tcgen05)
  d |= (uint64_t)2 << 61;                          // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor for kind::f16: D=f32, A/B = bf16 or f16, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_f16(bool bf16, int m, int n) {
  return (1u << 4)                                    // D format: f32
         | ((bf16 ? 1u : 0u) << 7)                    // A format
         | ((bf16 ? 1u : 0u) << 10)                   // B format
         | ((uint32_t)(n >> 3) << 17)                 // N / 8
         | ((uint32_t)(m >> 4) << 24);                // M / 16
}

__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace oc
