// Decode-sized (M <= 16) GPTQ int4 GEMV on the 5th-generation tensor cores (tcgen05), for
// uniform groups of 32, 64 or a multiple of 64 rows.
//
// Replaces the small-M launches of the reference's Triton kernel (fused_int4_linear.py:127-272)
// and PackedGPTQLinear's dequant + F.linear (packed_gptq_linear.py:66-74) for decode.
//
// Why tcgen05 here: the legacy mma.sync pipe of sm_100 peaks near 550 TFLOP/s, and a decode
// GEMV streaming int4 weights at HBM speed needs about half of it for the MMAs alone. On the
// 5th-generation tensor cores an MMA of 128 features x 16 tokens x 16 k costs a few cycles, so
// the kernel is left with the nibble extraction and the memory streams.
//
// Factored scaling (as in gemv.cuh): the A operand is the raw magic-biased codes (M + q),
// exact in bf16/fp16, written by the dequant warpgroups into TMEM (128 lanes = 128 features);
// the B operand is the activation block [16 tokens x 64 k] (TMA, 128-byte swizzle, rows past M
// zero). Per group the MMA accumulates D = sum_k (M + q) x into a TMEM buffer and, with an
// all-ones A operand, S = sum_k x; flush warps apply
//     sum_k x s (q - z) = s D - s (M + z) S
// in fp32 per group and accumulate in registers. Group buffers rotate through 8 TMEM slots so
// the MMAs of the next groups proceed while a group is flushed.
//
// Warp roles (512 threads, one CTA per SM, one 128-feature tile and one K range per CTA):
//   warp 0 lane 0: activation TMA producer (after griddepcontrol.wait)
//   warp 2 lane 0: packed-weight and per-group scale/zero TMA producer (before the wait)
//   warp 1: TMEM alloc + MMA issuer (lane 0)
//   warps 4-7 / 8-11: nibble-to-code warpgroups for even / odd 64-k blocks (tcgen05.st)
//   warps 12-15: group flush + split-K reduction + epilogue
// Launched with programmatic stream serialization (see gemv_tma.cuh). Every mbarrier wait is
// bounded; on timeout the kernel records an error code, drains its own copies / MMAs, frees
// TMEM and skips its global writes.
#pragma once

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_tma.cuh"

namespace oc {

constexpr int kVtThreads = 512;
constexpr int kVtBK = 64;         // k per stage
constexpr int kVtN = 16;          // MMA N: tokens (M <= 16, rows past M are zero)
constexpr int kVtWS = 24;         // packed-weight stages (8 rows x 128 words = 4 KB each)
constexpr int kVtXS = 8;          // activation stages ([16 tokens x 64 k] = 2 KB each)
constexpr int kVtSZ = 16;         // per-group scale/zero stages
constexpr int kVtAS = 6;          // TMEM A stages (32 columns each)
constexpr int kVtND = 8;          // TMEM group buffers (16 columns for D, 16 for S)
constexpr int kVtWBytes = 8 * kGemvCols * 4;
constexpr int kVtXBytes = kVtN * kVtBK * 2;
constexpr int kVtSZBytes = 384;   // 128 scales (256 B) + 16 zero words (64 B), 128-B aligned
constexpr int kVtColOnes = kVtAS * 32;          // 192: all-ones A tile (8 columns)
constexpr int kVtColD = 256;                    // D buffers: 256 + 16 db
constexpr int kVtColS = 384;                    // S buffers: 384 + 16 db
constexpr int kVtXOff = 0;
constexpr int kVtWOff = kVtXOff + kVtXS * kVtXBytes;
constexpr int kVtSZOff = kVtWOff + kVtWS * kVtWBytes;
constexpr int kVtBarOff = kVtSZOff + kVtSZ * kVtSZBytes;
constexpr int kVtNumBars = 2 * (kVtWS + kVtXS + kVtAS + kVtSZ + kVtND) + 1;
constexpr int kVtSmemBytes = kVtBarOff + kVtNumBars * 8 + 16 + 1024 /*align*/;
static_assert(kVtSmemBytes <= 232448, "shared memory per CTA");

struct VtParams {
  GemvParams g;
  int kb_per_split;  // 64-k blocks per split
};

template <bool BF16>
__global__ void __launch_bounds__(kVtThreads, 1)
    gptq_gemv_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_s1,
                        const __grid_constant__ CUtensorMap tmap_z1, const __grid_constant__ CUtensorMap tmap_x,
                        const VtParams vp) {
  using P = Pair<BF16>;
  const GemvParams& p = vp.g;
  extern __shared__ __align__(1024) uint8_t vt_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(vt_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kVtBarOff);
  uint64_t* full_w = bars;
  uint64_t* empty_w = full_w + kVtWS;
  uint64_t* full_x = empty_w + kVtWS;
  uint64_t* empty_x = full_x + kVtXS;
  uint64_t* full_a = empty_x + kVtXS;
  uint64_t* empty_a = full_a + kVtAS;
  uint64_t* full_sz = empty_a + kVtAS;
  uint64_t* empty_sz = full_sz + kVtSZ;
  uint64_t* dfull = empty_sz + kVtSZ;
  uint64_t* dempty = dfull + kVtND;
  uint64_t* drain = dempty + kVtND;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  __shared__ int is_last;

  const int warp = warp_id(), lane = lane_id();
  const int tile = blockIdx.x, split = blockIdx.y;
  const int col0 = tile * kGemvCols;
  const int KB = (p.Kp + kVtBK - 1) / kVtBK;
  const int kb0 = split * vp.kb_per_split;
  const int kb1 = min(KB, kb0 + vp.kb_per_split);
  const int nkb = kb1 - kb0;
  const int gsteps = p.gs / 16;                   // 16-k MMA steps per group
  const int g_first = (kb0 * kVtBK) / p.gs;       // groups this CTA touches: g_first .. g_last
  const int g_last = (kb1 * kVtBK - 1) / p.gs;
  const int ngroups = g_last - g_first + 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kVtWS; ++i) { mbar_init(&full_w[i], 1); mbar_init(&empty_w[i], 128); }
    for (int i = 0; i < kVtXS; ++i) { mbar_init(&full_x[i], 1); mbar_init(&empty_x[i], 1); }
    for (int i = 0; i < kVtAS; ++i) { mbar_init(&full_a[i], 128); mbar_init(&empty_a[i], 1); }
    for (int i = 0; i < kVtSZ; ++i) { mbar_init(&full_sz[i], 1); mbar_init(&empty_sz[i], 128); }
    for (int i = 0; i < kVtND; ++i) { mbar_init(&dfull[i], 1); mbar_init(&dempty[i], 128); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  griddep_launch_dependents();

  // the all-ones A tile (16 k x 128 rows) used for the activation sums
  if (warp >= 4 && warp < 8) {
    const uint32_t one2 = BF16 ? 0x3F803F80u : 0x3C003C00u;
    const uint32_t r8[8] = {one2, one2, one2, one2, one2, one2, one2, one2};
    tmem_st_32x32b_x8(tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + kVtColOnes, r8);
    tc_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    // ------------------------------------------------------------------ activation producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      griddep_wait();  // x is written by the previous kernel
      int armed[kVtXS];
      for (int i = 0; i < kVtXS; ++i) armed[i] = -1;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % kVtXS, ph = (i / kVtXS) & 1;
        if (!mbar_wait(&empty_x[s], ph ^ 1, abort_flag, kDevErrTmaEmpty)) break;
        mbar_arrive_expect_tx(&full_x[s], kVtXBytes);
        tma_load_2d(smem + kVtXOff + s * kVtXBytes, &tmap_x, &full_x[s], (kb0 + i) * kVtBK, 0);
        armed[s] = ph;
      }
      // every copy issued lands before the CTA can exit (consumed ones return at once)
      for (int s = 0; s < kVtXS; ++s)
        if (armed[s] >= 0) mbar_drain(&full_x[s], armed[s]);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ weight / scale producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_s1);
      tma_prefetch_desc(&tmap_z1);
      int warmed[kVtWS], zarmed[kVtSZ];
      for (int i = 0; i < kVtWS; ++i) warmed[i] = -1;
      for (int i = 0; i < kVtSZ; ++i) zarmed[i] = -1;
      bool ok = true;
      int gi = 0;  // next group (sequence index) whose scales are due
      for (int i = 0; ok && i < nkb; ++i) {
        const int kb = kb0 + i;
        // scales / zeros of every group that starts inside this block (or the range's first)
        const int glast_here = (kb * kVtBK + kVtBK - 1) / p.gs;
        for (; gi <= glast_here - g_first; ++gi) {
          const int s = gi % kVtSZ, ph = (gi / kVtSZ) & 1;
          if (!mbar_wait(&empty_sz[s], ph ^ 1, abort_flag, kDevErrWEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_sz[s], kGemvCols * 2 + (kGemvCols / 8) * 4);
          tma_load_2d(smem + kVtSZOff + s * kVtSZBytes, &tmap_s1, &full_sz[s], col0, g_first + gi);
          tma_load_2d(smem + kVtSZOff + s * kVtSZBytes + 256, &tmap_z1, &full_sz[s], col0 / 8, g_first + gi);
          zarmed[s] = ph;
        }
        if (!ok) break;
        const int s = i % kVtWS, ph = (i / kVtWS) & 1;
        if (!mbar_wait(&empty_w[s], ph ^ 1, abort_flag, kDevErrWEmpty)) { ok = false; break; }
        mbar_arrive_expect_tx(&full_w[s], kVtWBytes);
        tma_load_2d(smem + kVtWOff + s * kVtWBytes, &tmap_w, &full_w[s], col0, kb * 8);
        warmed[s] = ph;
      }
      // every copy issued lands before the CTA can exit (consumed ones return at once)
      for (int s = 0; s < kVtWS; ++s)
        if (warmed[s] >= 0) mbar_drain(&full_w[s], warmed[s]);
      for (int s = 0; s < kVtSZ; ++s)
        if (zarmed[s] >= 0) mbar_drain(&full_sz[s], zarmed[s]);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BF16, kGemvCols, kVtN);
      bool ok = true, issued = false;
      int gi = 0, pos = (kb0 * 4) % gsteps;  // group sequence index, step within the group
      bool grp_open = false;
      uint32_t dcol = 0, scol = 0;
      uint32_t acc_flag = 0;
      for (int i = 0; ok && i < nkb; ++i) {
        const int sx = i % kVtXS, px = (i / kVtXS) & 1;
        const int sa = i % kVtAS, pa = (i / kVtAS) & 1;
        if (!mbar_wait(&full_x[sx], px, abort_flag, kDevErrTmaFull)) { ok = false; break; }
        if (!mbar_wait(&full_a[sa], pa, abort_flag, kDevErrAFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t xaddr = smem_u32(smem + kVtXOff + sx * kVtXBytes);
        const uint32_t a_tmem = tmem_base + (uint32_t)(sa * 32);
#pragma unroll 1
        for (int j = 0; j < kVtBK / 16; ++j) {
          if (!grp_open) {  // first step of a group: wait until its buffer has been flushed
            const int db = gi % kVtND;
            if (!mbar_wait(&dempty[db], ((gi / kVtND) & 1) ^ 1, abort_flag, kDevErrAccEmpty)) {
              ok = false;
              break;
            }
            tc_fence_after();
            dcol = tmem_base + kVtColD + db * 16;
            scol = tmem_base + kVtColS + db * 16;
            acc_flag = 0;
            grp_open = true;
          }
          const uint64_t bdesc = smem_desc_kmajor_sw128(xaddr + j * 32);
          tc_mma_ts(dcol, a_tmem + j * 8, bdesc, idesc, acc_flag);
          tc_mma_ts(scol, tmem_base + kVtColOnes, bdesc, idesc, acc_flag);
          issued = true;
          acc_flag = 1;
          const bool last_step = (i == nkb - 1) && (j == kVtBK / 16 - 1);
          if (++pos == gsteps || last_step) {
            tc_commit(&dfull[gi % kVtND]);
            ++gi;
            pos = 0;
            grp_open = false;
          }
        }
        if (!ok) break;
        tc_commit(&empty_x[sx]);
        tc_commit(&empty_a[sa]);
      }
      if (!ok && issued) {
        tc_commit(drain);
        mbar_drain(drain, 0);
      }
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------------ nibble-to-code warpgroups
    using Pp = Pair<BF16>;
    const int wg = (warp - 4) >> 2;
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    for (int i = wg; i < nkb; i += 2) {
      const int sw = i % kVtWS, pw = (i / kVtWS) & 1;
      const int sa = i % kVtAS, pa = (i / kVtAS) & 1;
      if (!mbar_wait(&full_w[sw], pw, abort_flag, kDevErrWFull)) break;
      const uint32_t* wt = reinterpret_cast<const uint32_t*>(smem + kVtWOff + sw * kVtWBytes);
      uint32_t q[8];
#pragma unroll
      for (int w = 0; w < 8; ++w) q[w] = wt[w * kGemvCols + row];
      mbar_arrive(&empty_w[sw]);
      uint32_t r32[32];
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const uint32_t p0 = lop3_and_or(q[w], 0x000F000Fu, Pp::kMagic);        // k0,k4
        const uint32_t p1 = lop3_and_or(q[w] >> 4, 0x000F000Fu, Pp::kMagic);   // k1,k5
        const uint32_t p2 = lop3_and_or(q[w] >> 8, 0x000F000Fu, Pp::kMagic);   // k2,k6
        const uint32_t p3 = lop3_and_or(q[w] >> 12, 0x000F000Fu, Pp::kMagic);  // k3,k7
        r32[4 * w + 0] = prmt(p0, p1, 0x5410u);  // k0,k1
        r32[4 * w + 1] = prmt(p2, p3, 0x5410u);  // k2,k3
        r32[4 * w + 2] = prmt(p0, p1, 0x7632u);  // k4,k5
        r32[4 * w + 3] = prmt(p2, p3, 0x7632u);  // k6,k7
      }
      if (!mbar_wait(&empty_a[sa], pa ^ 1, abort_flag, kDevErrAEmpty)) break;
      tc_fence_after();
      __syncwarp();
      tmem_st_32x32b_x32(tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(sa * 32), r32);
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&full_a[sa]);
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------------ group flush + epilogue
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const int n = col0 + row;
    const int et = threadIdx.x - 12 * 32;
    const int zsh = 4 * (n & 7);
    float acc[kVtN];
#pragma unroll
    for (int t = 0; t < kVtN; ++t) acc[t] = 0.f;
    bool ok = true;
    for (int gi = 0; gi < ngroups; ++gi) {
      const int ss = gi % kVtSZ;
      if (!mbar_wait(&full_sz[ss], (gi / kVtSZ) & 1, abort_flag, kDevErrWFull)) { ok = false; break; }
      const uint8_t* sz = smem + kVtSZOff + ss * kVtSZBytes;
      const uint16_t sbits = reinterpret_cast<const uint16_t*>(sz)[row];
      const uint32_t zw = reinterpret_cast<const uint32_t*>(sz + 256)[row >> 3];
      mbar_arrive(&empty_sz[ss]);
      uint32_t z = (zw >> zsh) & 0xFu;
      if (p.v1) z = (z + 1u) & 0xFu;
      const float sc = (p.s_dtype == kF16) ? __half2float(__ushort_as_half(sbits))
                                           : __bfloat162float(__ushort_as_bfloat16(sbits));
      const float cz = sc * (P::kMagicF + (float)z);  // exact: <= 19 significant bits
      const int db = gi % kVtND;
      if (!mbar_wait(&dfull[db], (gi / kVtND) & 1, abort_flag, kDevErrAccFull)) { ok = false; break; }
      tc_fence_after();
      uint32_t dv[16], sv[16];
      const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
      tmem_ld_32x32b_x16(tmem_base + lane_off + kVtColD + db * 16, dv);
      tmem_ld_32x32b_x16(tmem_base + lane_off + kVtColS + db * 16, sv);
      tc_wait_ld();
      tc_fence_before();
      mbar_arrive(&dempty[db]);
#pragma unroll
      for (int t = 0; t < kVtN; ++t) acc[t] = fmaf(sc, __uint_as_float(dv[t]), fmaf(-cz, __uint_as_float(sv[t]), acc[t]));
    }
    const bool any_fail = named_bar_or(1, 128, !ok);
    griddep_wait();  // the previous kernel is done with the workspace and the output
    const bool nvalid = n < p.N;
    {
      // a failed CTA (its error is recorded) still takes its split-K ticket and writes nothing;
      // the last CTA re-arms the ticket and skips the output if any split failed
      if (p.splits > 1) {
        if (!any_fail && nvalid)
          for (int t = 0; t < p.M; ++t) p.ws[((long long)split * p.M + t) * p.N + n] = acc[t];
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) {
          const unsigned prev = atomicAdd(p.tickets + tile, any_fail ? 1u + kTicketFail : 1u);
          const bool last = (prev & (kTicketFail - 1u)) == (unsigned)(p.splits - 1);
          is_last = !last ? 0 : ((prev >= kTicketFail || any_fail) ? 2 : 1);
          if (last) p.tickets[tile] = 0u;  // re-arm for the next launch (stream order)
        }
        named_bar_sync(1, 128);
        if (is_last == 1) {
          __threadfence();
          if (nvalid)
            for (int t = 0; t < p.M; ++t) {
              float sum = 0.f;
              for (int sp = 0; sp < p.splits; ++sp) sum += __ldcg(p.ws + ((long long)sp * p.M + t) * p.N + n);
              acc[t] = sum;
            }
        }
      }
      if (((p.splits == 1 && !any_fail) || (p.splits > 1 && is_last == 1)) && nvalid) {
        const int odt = BF16 ? kBF16 : kF16;
        const float bv = p.bias ? load_as_f32(p.bias, p.bias_dtype, n) : 0.f;
#pragma unroll
        for (int t = 0; t < kVtN; ++t)
          if (t < p.M) {
            const uint16_t* res = p.residual ? p.residual + (long long)t * p.ldr + n : nullptr;
            p.out[(long long)t * p.ldc + n] = f32_to_bits(epilogue_value(acc[t], bv, p.act, res, odt), odt);
          }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace oc
