// All-reduce (sum) of a bf16 buffer through NVLink SHARP (NVLS): the tensor-parallel reduction
// after each row-parallel linear of the sharded DiT stack. The reference has no distributed code;
// this replaces the NCCL all-reduce the row-parallel layer would otherwise call.
//
// The buffer is one NVLink multicast object: every rank of the job holds its own copy, and an
// access through the multicast address goes to every copy at once. Each rank reduces one slice
// (1/world of the range): multimem.ld_reduce reads the slice from all copies and the switch
// returns their sum (the switch's own bf16 addition: within one bf16 unit in the last place of the
// exact sum, not always the nearest value), multimem.st writes the sum back
// to all copies. Per rank that is the slice in and out once, against the 2 (world-1)/world of the
// whole buffer a ring all-reduce moves.
//
// Ordering. Before reading, every rank must have finished writing its copy (the GEMM that
// produced it ran earlier in that rank's stream); before anyone reads the result or overwrites
// its copy for the next chunk, every rank's stores must have landed. Two barriers give this: each
// block stores `epoch` with release semantics into its slot in every rank's flag array, then
// waits (acquire, bounded) until every rank's block with the same index has done the same in its
// own array. Flags are epochs that only grow, so the arrays are never reset between calls.
// A wait that runs out records kDevErrPeer and the kernel returns without writing.
#pragma once

#include "common.cuh"

namespace oc {

constexpr int kArMaxWorld = 8;
constexpr int kArMaxBlocks = 64;
constexpr int kArThreads = 512;
constexpr unsigned kDevErrPeer = 0x110;

struct ArParams {
  uint4* mc;                // multicast address of the first 16-byte vector of the range
  long long n16;            // 16-byte vectors in the range
  uint32_t* const* flags;   // [world] device-visible pointers to each rank's flag array
  int rank, world;
  uint32_t epoch;           // this call's epoch (> every earlier call's)
  unsigned long long wait_ns;
};

// Flag slot of (phase, block, source rank) in a flag array of [2][gridDim.x][world] words.
__device__ __forceinline__ int ar_slot(int phase, int block, int src, int world, int blocks) {
  return (phase * blocks + block) * world + src;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Cross-rank barrier of this block: returns false (error recorded) if some rank did not arrive
// within the wait bound. Every thread of the block returns the same value.
__device__ __forceinline__ bool ar_barrier(const ArParams& p, int phase, int* ok_smem) {
  if (threadIdx.x == 0) *ok_smem = 1;
  __syncthreads();
  if (threadIdx.x < p.world) {
    const int t = threadIdx.x;
    __threadfence_system();  // this rank's earlier writes (and this block's stores) before the flag
    st_release_sys(p.flags[t] + ar_slot(phase, blockIdx.x, p.rank, p.world, gridDim.x), p.epoch);
    const uint32_t* mine = p.flags[p.rank] + ar_slot(phase, blockIdx.x, t, p.world, gridDim.x);
    if ((int)(ld_acquire_sys(mine) - p.epoch) < 0) {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t it = 1;; ++it) {
        if ((int)(ld_acquire_sys(mine) - p.epoch) >= 0) break;
        if ((it & 63u) == 0u && global_timer_ns() - t0 > p.wait_ns) {
          record_error(kDevErrPeer);
          *ok_smem = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return *ok_smem != 0;
}

__global__ void __launch_bounds__(kArThreads) nvls_allreduce_bf16_kernel(const ArParams p) {
  __shared__ int ok_smem;
  if (!ar_barrier(p, 0, &ok_smem)) return;  // every rank's copy is complete
  const long long per = (p.n16 + p.world - 1) / p.world;
  const long long lo = (long long)p.rank * per;
  const long long hi = min(p.n16, lo + per);
  const long long step = (long long)gridDim.x * blockDim.x;
  long long i = lo + (long long)blockIdx.x * blockDim.x + threadIdx.x;
  // eight vectors in flight per thread
  for (; i + 7 * step < hi; i += 8 * step) {
    uint32_t v[8][4];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                   : "=r"(v[u][0]), "=r"(v[u][1]), "=r"(v[u][2]), "=r"(v[u][3])
                   : "l"(p.mc + i + u * step)
                   : "memory");
#pragma unroll
    for (int u = 0; u < 8; ++u)
      asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(p.mc + i + u * step),
                   "r"(v[u][0]), "r"(v[u][1]), "r"(v[u][2]), "r"(v[u][3])
                   : "memory");
  }
  for (; i < hi; i += step) {
    uint32_t a, b, c, d;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
                 : "l"(p.mc + i)
                 : "memory");
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(p.mc + i), "r"(a), "r"(b),
                 "r"(c), "r"(d)
                 : "memory");
  }
  ar_barrier(p, 1, &ok_smem);  // every rank's stores have landed before anyone reads or rewrites
}

// ---- all-reduce + RMS norm ---------------------------------------------------------------------
// The DiT block normalizes each row-parallel output right after its all-reduce. Run separately,
// every rank normalizes every row of the reduced buffer (the norm is replicated N times). Here the
// ranks split the ROWS instead of the byte range: a warp reads one row of its rank's share through
// the switch (multimem.ld_reduce: the bf16 sum over the ranks), computes its mean square in fp32,
// scales it by rsqrt(mean + eps) (times an optional per-column gain) and multimem.st's the
// normalized row to every rank's copy. Same barriers and flag slots as the plain kernel, so both
// share one flag array and one epoch sequence.
constexpr int kArNormThreads = 384;  // 12 warps; a 4096-wide row per warp fits the 168 registers this allows
constexpr int kArNormMaxVpl = 16;  // 16-byte vectors per lane: rows up to 16 * 32 * 8 = 4096 columns

struct ArNormParams {
  ArParams ar;           // ar.mc = row 0 of the range; ar.n16 unused
  int rows, cols;        // rows stored contiguously (stride cols), cols % 8 == 0
  const uint4* gain;     // optional [cols] bf16 per-column gain, nullptr: none
  float eps;
};

template <int VPL>
__global__ void __launch_bounds__(kArNormThreads) nvls_allreduce_rmsnorm_bf16_kernel(const ArNormParams p) {
  __shared__ int ok_smem;
  if (!ar_barrier(p.ar, 0, &ok_smem)) return;  // every rank's copy is complete
  const int per = (p.rows + p.ar.world - 1) / p.ar.world;
  const int lo = p.ar.rank * per;
  const int hi = min(p.rows, lo + per);
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int nvec = p.cols >> 3;
  for (int row = lo + blockIdx.x * wpb + (threadIdx.x >> 5); row < hi; row += gridDim.x * wpb) {
    uint4* r = p.ar.mc + (long long)row * nvec;
    uint32_t v[VPL][4];
#pragma unroll
    for (int u = 0; u < VPL; ++u) {
      if (lane + 32 * u < nvec) {
        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v[u][0]), "=r"(v[u][1]), "=r"(v[u][2]), "=r"(v[u][3])
                     : "l"(r + lane + 32 * u)
                     : "memory");
      } else {
        v[u][0] = v[u][1] = v[u][2] = v[u][3] = 0u;
      }
    }
    // mean square of the reduced (bf16) row in fp32, as a norm applied after the all-reduce sees it
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < VPL; ++u)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = __uint_as_float(v[u][j] << 16), b = __uint_as_float(v[u][j] & 0xFFFF0000u);
        ss = fmaf(a, a, ss);
        ss = fmaf(b, b, ss);
      }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    const float rs = rsqrtf(ss / (float)p.cols + p.eps);
#pragma unroll
    for (int u = 0; u < VPL; ++u) {
      const int c = lane + 32 * u;
      if (c >= nvec) continue;
      uint32_t gw[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};  // bf16 pairs of 1.0
      if (p.gain) {
        const uint4 g = __ldg(p.gain + c);
        gw[0] = g.x; gw[1] = g.y; gw[2] = g.z; gw[3] = g.w;
      }
      uint32_t y[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = __uint_as_float(v[u][j] << 16) * rs, b = __uint_as_float(v[u][j] & 0xFFFF0000u) * rs;
        y[j] = pack2_rn<true>(a * __uint_as_float(gw[j] << 16), b * __uint_as_float(gw[j] & 0xFFFF0000u));
      }
      asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(r + c), "r"(y[0]),
                   "r"(y[1]), "r"(y[2]), "r"(y[3])
                   : "memory");
    }
  }
  ar_barrier(p.ar, 1, &ok_smem);  // every rank's stores have landed before anyone reads or rewrites
}

}  // namespace oc
