// Prefill / large-M int4 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Replaces the Triton kernel _fused_int4_gemm_kernel (fused_int4_linear.py:127-272) and
// its odd-group / any-group variants (:275-385, :540-636).
//
// Orientation: C^T tile = W_tile (128 output features) x X_tile^T (BT tokens).
//   * A operand = dequantized weights, written by the dequant warpgroups straight
//     into TMEM (tcgen05.st) -- 128 lanes = 128 output features, 2 bf16/fp16
//     per 32-bit column. The dequantized weights never touch shared memory.
//   * B operand = activation tile X[BT tokens, 64 k] loaded by TMA with the
//     128-byte swizzle (K-major canonical layout).
//   * D = fp32 accumulator in TMEM: 128 lanes x BT columns (tokens), double
//     buffered when TMEM allows so the epilogue overlaps the next tile.
//   * Per 64-k block a TMA stage carries the packed qweight tile [8 x 128] int32
//     and, for uniform aligned groups, the scale rows [R x 128] and zero rows
//     [R x 16 words] (R = 2 for groupsize 32, 1 for multiples of 64); other group
//     structures read scales/zeros with cached global loads.
//   * Exact dequant: w = RNE(s*(q-z)) as in quant_utils.dequant_gptq_to_fp.
//   * 8-bit layers (WB = 8, quant_utils.py:12-28 with wbits=8): a stage carries 16 word rows
//     (4 k per word); each code becomes the fp32 2^23 + q with one byte permute, q - z and
//     (q - z) * s are exact in fp32 (8 x 11 significant bits), and one conversion rounds a
//     pair to the activation dtype -- the reference's single rounding, for every scale dtype.
// Warp roles (512 threads, one persistent CTA per SM):
//   warp 0 lane 0: TMA producer of activation tiles
//   warp 2 lane 0: TMA producer of packed weights/scales/zeros (runs ahead, decoupled)
//   warp 1: TMEM alloc + MMA issuer (lane 0)
//   warps 4-7 / 8-11: dequant warpgroups for even / odd k-blocks
//   warps 12-15: epilogue warpgroup (tcgen05.ld, bias, round, store)
// Every mbarrier wait is bounded in time; on timeout the kernel records an error
// code, drains its own TMA loads / MMAs, frees TMEM and returns.
#pragma once

#include "common.cuh"

namespace oc {

struct TcParams {
  int M, N, Kp;
  const uint32_t* qz;      // [G, N/8]
  const void* s;           // [G, N]
  int s_dtype;
  const int32_t* wgrp;     // [Kp/8] or null
  int G, gs, v1;
  int sz_tma;              // scales/zeros staged by TMA (uniform, aligned groups)
  int sz_rows;             // scale rows per 64-k block when sz_tma (1 or 2)
  const void* bias;
  int bias_dtype;
  const uint16_t* residual;  // optional [M, ldr] added after the activation
  long long ldr;
  int act;                   // Act
  uint16_t* out;
  long long ldc;
  int tma_epi;               // 1: output (and residual) tiles move by TMA through shared memory
  int n_tiles_n, n_tiles_m, num_tiles;
};

constexpr int kTcDqGroups = 2;   // dequant warpgroups (k-block `it` goes to group it % kTcDqGroups)
constexpr int kTcThreads = 128 * (2 + kTcDqGroups);
constexpr int kTcEpiWarp0 = 4 + 4 * kTcDqGroups;
constexpr int kTcBK = 64;            // k per pipeline stage (one 128-byte swizzle atom of 16-bit)
constexpr int kTcBN = 128;           // output features per tile (= TMEM lanes = UMMA M)
// One weight stage (64 k): packed words [64 * WB / 32 rows][128], scale rows [2][128] 16-bit,
// zero rows [2][128 * WB / 32] int32.
template <int WB>
struct TcW {
  static constexpr int kRows = kTcBK * WB / 32;                 // word rows: 8 (4-bit) or 16 (8-bit)
  static constexpr int kWBytes = kRows * kTcBN * 4;
  static constexpr int kSOff = kWBytes;
  static constexpr int kZWords = kTcBN * WB / 32;               // zero words per row: 16 or 32
  static constexpr int kZOff = kSOff + 2 * kTcBN * 2;
  static constexpr int kStageBytes = kZOff + 2 * kZWords * 4 + 128;  // 4864 / 9088, multiples of 128
  static_assert(kStageBytes % 128 == 0, "stage alignment");
};
constexpr int kTcWBytes = TcW<4>::kWBytes;
constexpr int kTcSOff = TcW<4>::kSOff;
constexpr int kTcZOff = TcW<4>::kZOff;
constexpr int kTcWStageBytes = TcW<4>::kStageBytes;

constexpr int kTcEpiBufs = 4;                        // staging buffers per epilogue warp
constexpr int kTcWarpChunkBytes = 32 * 32 * 2;         // one warp's chunk: [32 tokens][32 features] 16-bit
constexpr int kTcChunkBytes = 4 * kTcWarpChunkBytes;   // the four warps' buffers of one chunk slot

// BT tokens per MMA (UMMA N) and NSUB sub-tiles per tile: the NSUB sub-tiles of a tile share
// every dequantized weight stage, so the dequant work per MMA flop falls as 1 / (NSUB * BT).
// CG = 2: a cluster of two CTAs (one per SM) computes 256 features x the tile's tokens with
// cta_group::2 MMAs; each CTA dequantizes its own 128 features and holds half of every
// activation sub-tile (BT / 2 tokens), so the activation traffic per SM halves.
template <int BT, int NSUB, int ACC_STAGES, int X_STAGES, int W_STAGES, int A_STAGES, int CG = 1, int WB = 4>
struct TcCfg {
  static constexpr int kTileTok = NSUB * BT;
  static constexpr int kAccCols = ACC_STAGES * kTileTok;
  static constexpr int kACols = A_STAGES * (kTcBK / 2);
  static_assert(kAccCols + kACols <= 512, "TMEM budget");
  static_assert(BT % 32 == 0 && BT <= 256, "UMMA N");
  static_assert(CG == 1 || CG == 2, "CTA group");
  static constexpr int kXSubBytes = BT / CG * 128;  // this CTA's rows of one activation sub-tile
  static constexpr int kXStageBytes = NSUB * kXSubBytes;
  static constexpr int kEpiBytes = kTcEpiBufs * kTcChunkBytes;
  static constexpr int kSmemBytes = X_STAGES * kXStageBytes + W_STAGES * TcW<WB>::kStageBytes + kEpiBytes +
                                    1024 /*align*/ +
                                    (2 * (X_STAGES + W_STAGES + A_STAGES + ACC_STAGES) + 2 + 4 * kTcEpiBufs) * 8 + 64;
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

// One 32-token chunk of a warp's epilogue, specialised on the activation and the residual so
// the per-value loop carries no runtime tests: e[i * 32] (token i, this lane's feature) holds the
// residual on entry when RES and the rounded output on exit.
template <bool GELU, bool RES, int ODT>
__device__ __forceinline__ void epi_chunk(const uint32_t (&v)[32], float bv, uint16_t* e) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float o = __uint_as_float(v[i]) + bv;
    if constexpr (GELU) o = gelu_tanh(o);
    if constexpr (RES) o += bits_to_f32(e[i * 32], ODT);
    e[i * 32] = f32_to_bits(o, ODT);
  }
}

template <bool BF16, bool HAS_LO, int BT, int NSUB, int ACC_STAGES, int X_STAGES, int W_STAGES, int A_STAGES,
          int CG, int WB = 4>
__global__ void __launch_bounds__(kTcThreads, 1)
    gptq_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_s, const __grid_constant__ CUtensorMap tmap_z,
                        const __grid_constant__ CUtensorMap tmap_c, const __grid_constant__ CUtensorMap tmap_r,
                        const TcParams p) {
  using Cfg = TcCfg<BT, NSUB, ACC_STAGES, X_STAGES, W_STAGES, A_STAGES, CG, WB>;
  using WL = TcW<WB>;
  static_assert(WB == 4 || (WB == 8 && CG == 1), "8-bit codes: single CTAs");
  constexpr int kTileTok = Cfg::kTileTok;
  // CTA pairs: rank 0 (leader) issues the MMAs and owns the full_x / full_a / empty_acc
  // barriers the pair waits on; both CTAs own their empty_x / empty_a / full_acc barriers,
  // which the leader's commits reach by multicast.
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int tile0 = blockIdx.x / CG, tile_step = gridDim.x / CG;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* x_smem = smem;
  uint8_t* w_smem = x_smem + X_STAGES * Cfg::kXStageBytes;
  uint8_t* epi_smem = w_smem + W_STAGES * WL::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + Cfg::kEpiBytes);
  uint64_t* full_x = bars;
  uint64_t* empty_x = full_x + X_STAGES;
  uint64_t* full_w = empty_x + X_STAGES;
  uint64_t* empty_w = full_w + W_STAGES;
  uint64_t* full_a = empty_w + W_STAGES;
  uint64_t* empty_a = full_a + A_STAGES;
  uint64_t* full_acc = empty_a + A_STAGES;
  uint64_t* empty_acc = full_acc + ACC_STAGES;
  uint64_t* drain = empty_acc + ACC_STAGES;
  uint64_t* res_full = drain + 1;  // [4 epilogue warps][kTcEpiBufs]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(res_full + 4 * kTcEpiBufs);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = warp_id(), lane = lane_id();
  const int KB = (p.Kp + kTcBK - 1) / kTcBK;
  const uint32_t w_tx = WL::kWBytes + (p.sz_tma ? p.sz_rows * (kTcBN * 2 + WL::kZWords * 4) : 0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < X_STAGES; ++i) { mbar_init(&full_x[i], 1); mbar_init(&empty_x[i], 1); }
    for (int i = 0; i < W_STAGES; ++i) { mbar_init(&full_w[i], 1); mbar_init(&empty_w[i], 128); }
    // pairs arrive once per warp from each CTA (4 warps x 2), single CTAs once per thread
    for (int i = 0; i < A_STAGES; ++i) { mbar_init(&full_a[i], CG == 2 ? 8 : 128); mbar_init(&empty_a[i], 1); }
    for (int i = 0; i < ACC_STAGES; ++i) { mbar_init(&full_acc[i], 1); mbar_init(&empty_acc[i], CG == 2 ? 8 : 128); }
    mbar_init(drain, 1);
    for (int i = 0; i < 4 * kTcEpiBufs; ++i) mbar_init(&res_full[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
    if (p.sz_tma) {
      tma_prefetch_desc(&tmap_s);
      tma_prefetch_desc(&tmap_z);
    }
    if (p.tma_epi) tma_prefetch_desc(&tmap_c);
    if (p.tma_epi && p.residual) tma_prefetch_desc(&tmap_r);
  }
  if (warp == 1) {
    if (CG == 2) {
      tmem_alloc_cg2(tmem_holder, 512);
      tmem_relinquish_cg2();
    } else {
      tmem_alloc(tmem_holder, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (CG == 2)
    cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA arrive / copy
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer: activation tiles
    if (lane == 0) {
      int it = 0;
      int x_armed[X_STAGES];
      for (int i = 0; i < X_STAGES; ++i) x_armed[i] = -1;
      bool ok = true;
      for (int tile = tile0; ok && tile < p.num_tiles; tile += tile_step) {
        const int mb = tile / p.n_tiles_n;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int sx = it % X_STAGES, px = (it / X_STAGES) & 1;
          if (!mbar_wait(&empty_x[sx], px ^ 1, abort_flag, kDevErrTmaEmpty)) { ok = false; break; }
          if (CG == 2) {
            // both CTAs load their half of each sub-tile; the leader's barrier counts both
            if (leader) mbar_arrive_expect_tx(&full_x[sx], 2 * Cfg::kXStageBytes);
            const uint32_t bar = mapa_shared(&full_x[sx], 0);
#pragma unroll
            for (int sb = 0; sb < NSUB; ++sb)
              tma_load_2d_pair(x_smem + sx * Cfg::kXStageBytes + sb * Cfg::kXSubBytes, &tmap_x, bar, kb * kTcBK,
                               mb * kTileTok + sb * BT + (int)rank * (BT / 2));
          } else {
            mbar_arrive_expect_tx(&full_x[sx], Cfg::kXStageBytes);
#pragma unroll
            for (int sb = 0; sb < NSUB; ++sb)
              tma_load_2d(x_smem + sx * Cfg::kXStageBytes + sb * Cfg::kXSubBytes, &tmap_x, &full_x[sx], kb * kTcBK,
                          mb * kTileTok + sb * BT);
          }
          x_armed[sx] = px;
        }
      }
      if (CG == 2) {
        // Our loads signal the leader's barrier, so wait (bounded) until the pair's MMAs have
        // released every stage we filled: then each of our copies has landed.
        for (int i = 0; i < X_STAGES; ++i)
          if (x_armed[i] >= 0) mbar_drain(&empty_x[i], x_armed[i]);
      } else {
        // every load issued lands before the CTA (and its smem) can go away, whatever happened to
        // the other roles; loads already consumed have completed their phase and return at once
        for (int i = 0; i < X_STAGES; ++i)
          if (x_armed[i] >= 0) mbar_drain(&full_x[i], x_armed[i]);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ TMA producer: packed weights (+ scales/zeros)
    // Runs ahead of the activation stream by up to W_STAGES blocks so dequant overlaps the MMAs.
    if (lane == 0) {
      int it = 0;
      int w_armed[W_STAGES];
      for (int i = 0; i < W_STAGES; ++i) w_armed[i] = -1;
      bool ok = true;
      for (int tile = tile0; ok && tile < p.num_tiles; tile += tile_step) {
        const int nb = tile % p.n_tiles_n;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int sw = it % W_STAGES, pw = (it / W_STAGES) & 1;
          if (!mbar_wait(&empty_w[sw], pw ^ 1, abort_flag, kDevErrWEmpty)) { ok = false; break; }
          uint8_t* ws = w_smem + sw * WL::kStageBytes;
          mbar_arrive_expect_tx(&full_w[sw], w_tx);
          const int fb = nb * CG + (int)rank;  // this CTA's 128-feature block
          tma_load_2d(ws, &tmap_w, &full_w[sw], fb * kTcBN, kb * WL::kRows);
          if (p.sz_tma) {
            const int row0 = (p.sz_rows == 2) ? kb * 2 : (kb * kTcBK) / p.gs;
            tma_load_2d(ws + WL::kSOff, &tmap_s, &full_w[sw], fb * kTcBN, row0);
            tma_load_2d(ws + WL::kZOff, &tmap_z, &full_w[sw], fb * WL::kZWords, row0);
          }
          w_armed[sw] = pw;
        }
      }
      // every load issued lands before the CTA can exit (consumed ones return at once)
      for (int i = 0; i < W_STAGES; ++i)
        if (w_armed[i] >= 0) mbar_drain(&full_w[i], w_armed[i]);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_f16(BF16, kTcBN * CG, BT);
      int it = 0, tcount = 0;
      bool ok = true, issued = false;
      for (int tile = tile0; ok && tile < p.num_tiles; tile += tile_step, ++tcount) {
        const int sc = tcount % ACC_STAGES, pc = (tcount / ACC_STAGES) & 1;
        if (!mbar_wait(&empty_acc[sc], pc ^ 1, abort_flag, kDevErrAccEmpty)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(sc * kTileTok);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int sx = it % X_STAGES, px = (it / X_STAGES) & 1;
          const int sa = it % A_STAGES, pa = (it / A_STAGES) & 1;
          if (!mbar_wait(&full_x[sx], px, abort_flag, kDevErrTmaFull)) { ok = false; break; }
          if (!mbar_wait(&full_a[sa], pa, abort_flag, kDevErrAFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t xaddr = smem_u32(x_smem + sx * Cfg::kXStageBytes);
          const uint32_t a_tmem = tmem_base + (uint32_t)(Cfg::kAccCols + sa * (kTcBK / 2));
#pragma unroll
          for (int j = 0; j < kTcBK / 16; ++j)
#pragma unroll
            for (int sb = 0; sb < NSUB; ++sb) {
              const uint64_t bdesc = smem_desc_kmajor_sw128(xaddr + sb * Cfg::kXSubBytes + j * 32);
              if (CG == 2)
                tc_mma_ts_pair(d_tmem + sb * BT, a_tmem + j * 8, bdesc, idesc, (kb | j) != 0 ? 1u : 0u);
              else
                tc_mma_ts(d_tmem + sb * BT, a_tmem + j * 8, bdesc, idesc, (kb | j) != 0 ? 1u : 0u);
            }
          issued = true;
          if (CG == 2) {
            tc_commit_pair(&empty_x[sx], 0x3);
            tc_commit_pair(&empty_a[sa], 0x3);
          } else {
            tc_commit(&empty_x[sx]);
            tc_commit(&empty_a[sa]);
          }
        }
        if (!ok) break;
        if (CG == 2)
          tc_commit_pair(&full_acc[sc], 0x3);
        else
          tc_commit(&full_acc[sc]);
      }
      if (!ok && issued) {
        if (CG == 2)
          tc_commit_pair(drain, 0x1);
        else
          tc_commit(drain);
        mbar_drain(drain, 0);
      }
    }
  } else if (warp >= 4 && warp < kTcEpiWarp0) {
    // ------------------------------------------------------------ dequant warpgroups
    using Pp = Pair<BF16>;
    const int wg = (warp - 4) >> 2;   // takes k-blocks it with it % kTcDqGroups == wg
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;   // TMEM lane == output feature within the tile
    const int kw_rows = p.Kp >> 3;
    int it = 0;
    bool ok = true;
    for (int tile = tile0; ok && tile < p.num_tiles; tile += tile_step) {
      const int nb = tile % p.n_tiles_n;
      const int n = (nb * CG + (int)rank) * kTcBN + row;
      const int nn = n < p.N ? n : 0;
      const int zsh = 4 * (nn & 7);
      for (int kb = 0; kb < KB; ++kb, ++it) {
        if ((it % kTcDqGroups) != wg) continue;
        const int sw = it % W_STAGES, pw = (it / W_STAGES) & 1;
        const int sa = it % A_STAGES, pa = (it / A_STAGES) & 1;
        uint32_t r32[32];
        if constexpr (WB == 8) {
          // 16 words of 4 codes; uniform groups with scale / zero rows staged by TMA (the host
          // only builds 8-bit layers that way): row r covers words 8r .. 8r+7 when there are two
          if (!mbar_wait(&full_w[sw], pw, abort_flag, kDevErrWFull)) { ok = false; break; }
          const uint8_t* ws = w_smem + sw * WL::kStageBytes;
          const uint32_t* wt = reinterpret_cast<const uint32_t*>(ws);
          uint32_t q[16];
#pragma unroll
          for (int w = 0; w < 16; ++w) q[w] = wt[w * kTcBN + row];
          const uint16_t* st = reinterpret_cast<const uint16_t*>(ws + WL::kSOff);
          const uint32_t* zt = reinterpret_cast<const uint32_t*>(ws + WL::kZOff);
          float sr[2], zr[2];  // scale, 2^23 + z of the stage's (up to two) groups
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int rr = r < p.sz_rows ? r : 0;
            const uint16_t sb = st[rr * kTcBN + row];
            sr[r] = (p.s_dtype == kF16) ? __half2float(__ushort_as_half(sb)) : __bfloat162float(__ushort_as_bfloat16(sb));
            uint32_t z = (zt[rr * WL::kZWords + (row >> 2)] >> (8 * (row & 3))) & 0xFFu;
            if (p.v1) z = (z + 1u) & 0xFFu;
            zr[r] = 8388608.f + (float)z;
          }
          mbar_arrive(&empty_w[sw]);
#pragma unroll
          for (int w = 0; w < 16; ++w) {
            const float sv = (w >= 8) ? sr[1] : sr[0];
            const float zv = (w >= 8) ? zr[1] : zr[0];
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float qf = __uint_as_float(prmt(q[w], 0x4B000000u, 0x7540u | (uint32_t)j));  // 2^23 + q_j
              v[j] = __fmul_rn(__fsub_rn(qf, zv), sv);  // exact: (q - z) * s has <= 19 significant bits
            }
            r32[2 * w] = pack2_rn<BF16>(v[0], v[1]);      // k 4w, 4w+1
            r32[2 * w + 1] = pack2_rn<BF16>(v[2], v[3]);  // k 4w+2, 4w+3
          }
        } else {
          // per-word group constants. fp16 activations with bf16 scales (HAS_LO && !BF16) keep
          // each word's scale and zero too: a bf16 scale outside fp16's range makes the split
          // inexact, and then the warp's block takes the fp32 formula instead (below).
          constexpr bool kCheck = HAS_LO && !BF16;
          DqConst<BF16> cst[8];
          float sfw[kCheck ? 8 : 1];
          int zfw[kCheck ? 8 : 1];
          bool exact = true;
          if (!p.sz_tma) {
            int last = -1;
            float sv = 0.f;
            uint32_t zw = 0;
  #pragma unroll
            for (int w = 0; w < 8; ++w) {
              const int kw = kb * 8 + w;
              const int grp = (kw < kw_rows) ? (p.wgrp ? __ldg(p.wgrp + kw) : (8 * kw) / p.gs) : 0;
              if (grp != last) {
                sv = load_as_f32(p.s, p.s_dtype, (long long)grp * p.N + nn);
                zw = __ldg(p.qz + (long long)grp * (p.N >> 3) + (nn >> 3));
                uint32_t z = (zw >> zsh) & 0xFu;
                if (p.v1) z = (z + 1u) & 0xFu;
                cst[w] = make_dq_const<BF16>(sv, (int)z);
                if constexpr (kCheck) {
                  exact = exact && dq_const_exact<BF16>(sv, cst[w]);
                  sfw[w] = sv;
                  zfw[w] = (int)z;
                }
                last = grp;
              } else {
                cst[w] = cst[w > 0 ? w - 1 : 0];
                if constexpr (kCheck) {
                  sfw[w] = sfw[w > 0 ? w - 1 : 0];
                  zfw[w] = zfw[w > 0 ? w - 1 : 0];
                }
              }
            }
          }
          if (!mbar_wait(&full_w[sw], pw, abort_flag, kDevErrWFull)) { ok = false; break; }
          const uint8_t* ws = w_smem + sw * WL::kStageBytes;
          const uint32_t* wt = reinterpret_cast<const uint32_t*>(ws);
          uint32_t q[8];
  #pragma unroll
          for (int w = 0; w < 8; ++w) q[w] = wt[w * kTcBN + row];
          if (p.sz_tma) {
            const uint16_t* st = reinterpret_cast<const uint16_t*>(ws + kTcSOff);
            const uint32_t* zt = reinterpret_cast<const uint32_t*>(ws + kTcZOff);
            const int nr = p.sz_rows;
  #pragma unroll
            for (int r = 0; r < 2; ++r) {
              if (r < nr) {
                const float sv = (p.s_dtype == kF16) ? __half2float(__ushort_as_half(st[r * kTcBN + row]))
                                                     : __bfloat162float(__ushort_as_bfloat16(st[r * kTcBN + row]));
                uint32_t z = (zt[r * 16 + (row >> 3)] >> zsh) & 0xFu;
                if (p.v1) z = (z + 1u) & 0xFu;
                const DqConst<BF16> c = make_dq_const<BF16>(sv, (int)z);
                if constexpr (kCheck) exact = exact && dq_const_exact<BF16>(sv, c);
                // words 4r..4r+3 (nr == 2) or all 8 words (nr == 1)
  #pragma unroll
                for (int w = 0; w < 8; ++w)
                  if ((nr == 1) || (w >> 2) == r) {
                    cst[w] = c;
                    if constexpr (kCheck) {
                      sfw[w] = sv;
                      zfw[w] = (int)z;
                    }
                  }
              }
            }
          }
          mbar_arrive(&empty_w[sw]);

          if (!kCheck || __all_sync(0xffffffffu, exact)) {
  #pragma unroll
            for (int w = 0; w < 8; ++w) {
              const uint32_t qq = q[w];
              const uint32_t p0 = dq_pair<BF16, HAS_LO>(lop3_and_or(qq, 0x000F000Fu, Pp::kMagic), cst[w]);        // k0,k4
              const uint32_t p1 = dq_pair<BF16, HAS_LO>(lop3_and_or(qq >> 4, 0x000F000Fu, Pp::kMagic), cst[w]);   // k1,k5
              const uint32_t p2 = dq_pair<BF16, HAS_LO>(lop3_and_or(qq >> 8, 0x000F000Fu, Pp::kMagic), cst[w]);   // k2,k6
              const uint32_t p3 = dq_pair<BF16, HAS_LO>(lop3_and_or(qq >> 12, 0x000F000Fu, Pp::kMagic), cst[w]);  // k3,k7
              r32[4 * w + 0] = prmt(p0, p1, 0x5410u);  // k0,k1
              r32[4 * w + 1] = prmt(p2, p3, 0x5410u);  // k2,k3
              r32[4 * w + 2] = prmt(p0, p1, 0x7632u);  // k4,k5
              r32[4 * w + 3] = prmt(p2, p3, 0x7632u);  // k6,k7
            }
          } else if constexpr (kCheck) {
            // the formula of quant_utils.py:66-69 in fp32: (q - z) is an exact integer, its product
            // with a bf16 scale is exact in fp32, and one conversion rounds it to fp16
  #pragma unroll
            for (int w = 0; w < 8; ++w) {
              const uint32_t qq = q[w];
  #pragma unroll
              for (int j = 0; j < 8; j += 2) {
                const float da = (float)((int)((qq >> (4 * j)) & 0xFu) - zfw[w]);
                const float db = (float)((int)((qq >> (4 * j + 4)) & 0xFu) - zfw[w]);
                r32[4 * w + j / 2] = pack2_rn<BF16>(__fmul_rn(da, sfw[w]), __fmul_rn(db, sfw[w]));
              }
            }
          }
        }
        if (!mbar_wait(&empty_a[sa], pa ^ 1, abort_flag, kDevErrAEmpty)) { ok = false; break; }
        tc_fence_after();
        __syncwarp();
        const uint32_t taddr = tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(Cfg::kAccCols + sa * (kTcBK / 2));
        tmem_st_32x32b_x32(taddr, r32);
        tc_wait_st();
        tc_fence_before();
        if (CG == 2) {
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(&full_a[sa], 0));
        } else {
          mbar_arrive(&full_a[sa]);
        }
      }
    }
  } else if (warp >= kTcEpiWarp0 && p.tma_epi) {
    // ------------------------------------------------------------ epilogue warps, TMA path
    // Each of the four warps drains its 32 features (TMEM lanes) of the accumulator tile in
    // 32-token chunks through its own four staging buffers (running chunk counter q, buffer
    // q & 3), with no synchronisation across warps: lane 0 TMA-loads the residual chunk two
    // chunks ahead and TMA-stores each finished [32 x 32] chunk (rows past M and features past
    // N are clipped); bulk groups and residual barriers are per warp.
    const int q4 = warp & 3;
    constexpr int kChunks = kTileTok / 32;
    uint16_t* wepi = reinterpret_cast<uint16_t*>(epi_smem) + q4 * (kTcEpiBufs * kTcWarpChunkBytes / 2);
    uint64_t* wres = res_full + q4 * kTcEpiBufs;
    uint32_t q = 0;
    uint32_t res_pend = 0, res_par = 0;  // lane 0: buffers with a residual load in flight, its phase
    int tcount = 0;
    auto issue_res = [&](uint32_t qq, int f0, int m0) {  // lane 0
      const int b = qq & (kTcEpiBufs - 1);
      mbar_arrive_expect_tx(&wres[b], kTcWarpChunkBytes);
      tma_load_2d(wepi + b * (kTcWarpChunkBytes / 2), &tmap_r, &wres[b], f0, m0);
      res_pend |= 1u << b;
      res_par = (res_par & ~(1u << b)) | (((qq >> 2) & 1u) << b);
    };
    for (int tile = tile0; tile < p.num_tiles; tile += tile_step, ++tcount) {
      const int sc = tcount % ACC_STAGES, pc = (tcount / ACC_STAGES) & 1;
      const int nb = tile % p.n_tiles_n, mb = tile / p.n_tiles_n;
      const int f0 = (nb * CG + (int)rank) * kTcBN + q4 * 32;  // this warp's first feature
      const int n = f0 + lane;
      const int m_base = mb * kTileTok;
      const int nchunks = min(kChunks, (p.M - m_base + 31) / 32);  // chunks holding rows < M
      const float bv = (p.bias && n < p.N) ? load_as_f32(p.bias, p.bias_dtype, n) : 0.f;
      if (lane == 0) {
        bulk_wait_group_read<2>();  // stores q-3, q-4 have read buffers q, q+1
        if (p.residual)
          for (int c = 0; c < 2 && c < nchunks; ++c) issue_res(q + c, f0, m_base + c * 32);
      }
      __syncwarp();
      if (!mbar_wait(&full_acc[sc], pc, abort_flag, kDevErrAccFull)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(sc * kTileTok);
      bool failed = false;
#pragma unroll 1
      for (int c = 0; c < nchunks; ++c, ++q) {
        const int b = q & (kTcEpiBufs - 1);
        if (lane == 0 && c + 2 < nchunks) {
          bulk_wait_group_read<1>();  // store q-2 has read buffer q+2
          if (p.residual) issue_res(q + 2, f0, m_base + (c + 2) * 32);
        }
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), v);
        tc_wait_ld();
        if (p.residual) {
          if (!mbar_wait(&wres[b], (q >> 2) & 1, abort_flag, kDevErrResFull)) failed = true;
          if (__any_sync(0xffffffffu, failed)) {
            failed = true;
            break;
          }
          if (lane == 0) res_pend &= ~(1u << b);
        }
        __syncwarp();  // buffer b is free (lane 0 waited for its last store) / holds the residual
        uint16_t* e = wepi + b * (kTcWarpChunkBytes / 2) + lane;
        constexpr int kOdt = BF16 ? kBF16 : kF16;
        if (p.residual) {
          if (p.act == kActGeluTanh) epi_chunk<true, true, kOdt>(v, bv, e);
          else epi_chunk<false, true, kOdt>(v, bv, e);
        } else {
          if (p.act == kActGeluTanh) epi_chunk<true, false, kOdt>(v, bv, e);
          else epi_chunk<false, false, kOdt>(v, bv, e);
        }
        fence_proxy_async_shared();  // generic-proxy smem writes -> visible to the TMA store
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_c, wepi + b * (kTcWarpChunkBytes / 2), f0, m_base + c * 32);
          bulk_commit_group();
        }
      }
      if (failed) break;
      tc_fence_before();
      if (CG == 2) {  // this warp has read its accumulator lanes
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(&empty_acc[sc], 0));
      } else {
        mbar_arrive(&empty_acc[sc]);
      }
    }
    if (lane == 0) {
      bulk_wait_group0();
      for (int b = 0; b < kTcEpiBufs; ++b)  // residual loads issued ahead and never consumed
        if (res_pend & (1u << b)) mbar_drain(&wres[b], (res_par >> b) & 1u);
    }
  } else if (warp >= kTcEpiWarp0) {
    // ------------------------------------------------------------ epilogue warpgroup, direct stores
    // (outputs or residuals whose layout a tensor map cannot describe)
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const int odt = BF16 ? kBF16 : kF16;
    int tcount = 0;
    for (int tile = tile0; tile < p.num_tiles; tile += tile_step, ++tcount) {
      const int sc = tcount % ACC_STAGES, pc = (tcount / ACC_STAGES) & 1;
      const int nb = tile % p.n_tiles_n, mb = tile / p.n_tiles_n;
      const int n = (nb * CG + (int)rank) * kTcBN + row;
      const bool nvalid = n < p.N;
      const float bv = (p.bias && nvalid) ? load_as_f32(p.bias, p.bias_dtype, n) : 0.f;
      if (!mbar_wait(&full_acc[sc], pc, abort_flag, kDevErrAccFull)) break;
      tc_fence_after();
      __syncwarp();
      const uint32_t tbase = tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(sc * kTileTok);
#pragma unroll 1
      for (int c = 0; c < kTileTok / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), v);
        tc_wait_ld();
        const int m0 = mb * kTileTok + c * 32;
        if (nvalid) {
          uint16_t* dst = p.out + (long long)m0 * p.ldc + n;
          if (!p.residual && p.act == kActNone) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (m0 + i < p.M) dst[(long long)i * p.ldc] = f32_to_bits(__uint_as_float(v[i]) + bv, odt);
          } else {
            // residual rows first: 32 independent loads in flight, then the math and stores
            float rv[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) rv[i] = 0.f;
            if (p.residual) {
              const uint16_t* res = p.residual + (long long)m0 * p.ldr + n;
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (m0 + i < p.M) rv[i] = bits_to_f32(__ldg(res + (long long)i * p.ldr), odt);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (m0 + i < p.M) {
                float o = __uint_as_float(v[i]) + bv;
                if (p.act == kActGeluTanh) o = gelu_tanh(o);
                dst[(long long)i * p.ldc] = f32_to_bits(o + rv[i], odt);
              }
          }
        }
      }
      tc_fence_before();
      if (CG == 2) {
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(&empty_acc[sc], 0));
      } else {
        mbar_arrive(&empty_acc[sc]);
      }
    }
  }

  tc_fence_before();
  if (CG == 2)
    cluster_sync_all();  // neither CTA leaves (or frees TMEM) while the pair's MMAs / arrivals may touch it
  else
    __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if (CG == 2)
      tmem_dealloc_cg2(tmem_base, 512);
    else
      tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace oc
