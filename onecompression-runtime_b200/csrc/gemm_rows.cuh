// Row-packed int4/int2 GEMM on tcgen05 (sm_100a): RTN uint8-nibble layers, DSV4 int4/int2
// layers, and the grouped packed-expert GEMM of the MoE path.
//
// Replaces PackedRTNLinear.forward (packed_linear.py:53-56 -> quant_utils.py:72-103 + F.linear),
// Dsv4PackedLinear.forward (dsv4_packed_linear.py:95-98) and the per-expert loop over routed
// experts that the reference's DSV4 adapter runs (models/dsv4/loader.py:92-119).
//
// Weights: uint8 [N, ldq] per expert, 8/WBITS codes per byte along K (code j of a byte at
// bits j*WBITS; for WBITS = 4 the RTN layout "low nibble = even k" is the same thing).
// Scales/zeros: element (n, g) at n*stride_n + g*stride_g, any float dtype.
// Pipeline identical to gptq_gemm_tc_kernel (gemm_tc.cuh): dequantized weights are the
// MMA A operand in TMEM, activation tiles the B operand via TMA, fp32 accumulators in TMEM.
// Grouped mode: rows of X are sorted by expert, offsets[E+1] delimit the segments, and a
// tile never straddles two experts (the MMA may read rows of the next segment; those
// outputs are not stored).
// SwiGLU mode (SWIGLU): the expert FFN's gate and up projections in one launch. Each matrix is
// stored as [F, 2K] -- row n is gate row n followed by up row n (scales/zeros: the gate groups,
// then the up groups) -- so weight staging and dequant see an ordinary K' = 2K matrix. The
// activation k-block of step kb is kb mod K/64 (X is read twice per tile, the second time from
// L2), the MMA accumulates the first K/64 steps into the tile's gate accumulator and the rest into
// its up accumulator (two consecutive slots of the accumulator ring, each BT columns of the same
// TMEM lanes), and the epilogue writes silu(g) * u with g and u first rounded to the output type
// and silu_f32 as the silu-mul kernel computes it, so the bits equal separate gate / up GEMMs
// followed by that kernel: the [rows, 2F] intermediate and its extra pass disappear.
//
// Dequant numerics (MODE), bit-exact with the reference in every case:
//   kRowsExact   (DSV4, dsv4_packed_linear.py:52-56): w = RNE((q - z) * s) with the product in fp32.
//                 int2: a per-(row, group) table of the four weights, computed in fp32 and
//                 rounded once, indexed by the codes with byte permutes (any z and s).
//                 int4: pair arithmetic d = q - z, w = fma(d, s_hi, d * s_lo) when it is exact
//                 (half-integer zeros such as 1.5 or 7.5, 16-bit scales in range; checked per
//                 group, warp-uniformly), else the fp32 formula per weight.
//   kRowsRtn     (RTN, quant_utils.py:91-103): z_o = RNE(z), s_o = RNE(s),
//                 d = RNE(q - z_o), w = RNE(d * s_o) -- the reference's two roundings.
#pragma once

#include "common.cuh"

namespace oc {

enum RowsMode : int { kRowsExact = 0, kRowsRtn = 1 };

constexpr int kRowsMaxE = 1024;

struct RowsParams {
  int M;                      // dense: rows of X; grouped: total sorted rows
  int N, K;
  int E;                      // experts (1 = dense layer)
  const int32_t* offsets;     // [E+1] segment starts (grouped) or null (dense)
  const CUtensorMap* wmaps;   // [E] TMA maps over the packed weights (device memory)
  const void* const* sptr;    // [E] scales
  const void* const* zptr;    // [E] zeros
  const CUtensorMap* smaps;   // [E] TMA maps over scales / zeros stored [G, N] (sz_tma only)
  const CUtensorMap* zmaps;
  int kb_x;                   // SwiGLU mode: activation k-blocks (K / 2 / 64); else unused
  int s_dtype, z_dtype;
  long long s_stride_n, s_stride_g;
  int gs;                     // k per scale group (a multiple of the k held by one 32-bit word)
  int sz_tma;                 // scales/zeros ride in each weight stage by TMA
  int sz_rows;                // group rows per stage (64 / gs for small groups, else 1)
  int s_es, z_es;             // element bytes of scales / zeros
  const void* bias;
  int bias_dtype;
  uint16_t* out;
  long long ldc;
  int n_tiles_n;
};

// warps: 0 activation TMA, 1 MMA issuer, 2 weight TMA (and the m-tile prefix), 3 idle,
// 4 .. 4 + 4 kRowsDqGroups - 1 dequant warpgroups (k-block it goes to group it % kRowsDqGroups),
// the last 4 the epilogue
constexpr int kRowsDqGroups = 4;
constexpr int kRowsEpiWarp0 = 4 + 4 * kRowsDqGroups;
constexpr int kRowsThreads = 32 * (kRowsEpiWarp0 + 4);

template <int WBITS, int BT, int ACC_STAGES, int X_STAGES, int W_STAGES, int A_STAGES, bool SWIGLU = false>
struct RowsCfg {
  static constexpr int kKbBytes = 64 * WBITS / 8;               // packed bytes of one row per 64-k block
  static constexpr int kWBytes = 128 * kKbBytes;                 // 2 KB (int2) / 4 KB (int4)
  static constexpr int kSOff = kWBytes;                          // scale rows of the block (<= 512 B)
  static constexpr int kZOff = kWBytes + 512;                    // zero rows of the block (<= 512 B)
  static constexpr int kWStageBytes = kWBytes + 1024;
  static constexpr int kAccCols = ACC_STAGES * BT;              // a ring of BT-column accumulator slots
  static_assert(BT % 16 == 0 && (SWIGLU || BT % 32 == 0), "epilogue pieces: 16 tokens (SwiGLU), else 32");
  static constexpr int kACols = A_STAGES * 32;
  static_assert(kAccCols + kACols <= 512, "TMEM budget");
  static_assert(W_STAGES % kRowsDqGroups == 0 && A_STAGES % kRowsDqGroups == 0,
                "the dequant warpgroups take stages in turn");
  static constexpr int kXStageBytes = BT * 128;
  static constexpr int kSmemBytes = X_STAGES * kXStageBytes + W_STAGES * kWStageBytes + 1024 +
                                    (2 * (X_STAGES + W_STAGES + A_STAGES + ACC_STAGES) + 2) * 8 + 64 +
                                    (kRowsMaxE + 1) * 4;
  static_assert(kSmemBytes <= 232448, "shared memory per CTA");
};

template <bool BF16, int MODE>
struct RowsConst {
  uint32_t zm;   // (z, z) in the pair type (RNE of z)
  uint32_t zn;   // (-z, -z)
  uint32_t shi;  // RNE(s)
  uint32_t slo;  // exact mode: s - s_hi
};

template <bool BF16, int MODE>
__device__ __forceinline__ RowsConst<BF16, MODE> rows_const(float s, float z) {
  using P = Pair<BF16>;
  RowsConst<BF16, MODE> c;
  const uint16_t zz = P::from_f32(z);
  const uint16_t hi = P::from_f32(s);
  const uint16_t lo = P::from_f32(s - P::to_f32(hi));
  c.zm = pack2(zz, zz);
  c.zn = c.zm ^ 0x80008000u;
  c.shi = pack2(hi, hi);
  c.slo = pack2(lo, lo);
  return c;
}

// Exact mode: does the pair arithmetic give RNE_out(fp32((q - z) * s)) for every 4-bit code q?
// It does when z is a half-integer in [-1, 16] (then q - z has at most 5 significant bits, is
// exact in the pair type, and (q - z) * s is exact in fp32 for a 16-bit s) and the scale split is
// exact (split_exact). Other zeros and fp32 scales take the fp32 formula.
template <bool BF16, int MODE>
__device__ __forceinline__ bool rows_pair_exact(float s, float z, const RowsConst<BF16, MODE>& c) {
  using P = Pair<BF16>;
  const float z2 = 2.f * z;
  if (!(z2 == rintf(z2) && z >= -1.f && z <= 16.f)) return false;
  if (P::to_f32((uint16_t)(c.zm & 0xFFFFu)) != z) return false;
  return split_exact<BF16>(s, (uint16_t)(c.shi & 0xFFFFu), (uint16_t)(c.slo & 0xFFFFu));
}

// RNE(q - z) pair -> dequantized pair
template <bool BF16, int MODE, bool HAS_LO>
__device__ __forceinline__ uint32_t rows_scale(uint32_t d, const RowsConst<BF16, MODE>& c) {
  using P = Pair<BF16>;
  if (MODE == kRowsRtn) return P::mul(d, c.shi);
  if (HAS_LO) return P::fma(d, c.shi, P::mul(d, c.slo));
  return P::mul(d, c.shi);
}

// magic-biased code pair (M+c_a, M+c_b) -> dequantized pair
template <bool BF16, int MODE, bool HAS_LO>
__device__ __forceinline__ uint32_t rows_dq(uint32_t mq, const RowsConst<BF16, MODE>& c) {
  using P = Pair<BF16>;
  const uint32_t q = P::sub(mq, P::kMagic);   // exact integer codes
  const uint32_t d = P::sub(q, c.zm);         // RNE(q - z)
  return rows_scale<BF16, MODE, HAS_LO>(d, c);
}

template <bool BF16, int WBITS, int MODE, bool HAS_LO, int BT, int ACC_STAGES, int X_STAGES, int W_STAGES,
          int A_STAGES, bool SWIGLU = false>
__global__ void __launch_bounds__(kRowsThreads, 1)
    rows_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const RowsParams p) {
  using Cfg = RowsCfg<WBITS, BT, ACC_STAGES, X_STAGES, W_STAGES, A_STAGES, SWIGLU>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* x_smem = smem;
  uint8_t* w_smem = x_smem + X_STAGES * Cfg::kXStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_smem + W_STAGES * Cfg::kWStageBytes);
  uint64_t* full_x = bars;
  uint64_t* empty_x = full_x + X_STAGES;
  uint64_t* full_w = empty_x + X_STAGES;
  uint64_t* empty_w = full_w + W_STAGES;
  uint64_t* full_a = empty_w + W_STAGES;
  uint64_t* empty_a = full_a + A_STAGES;
  uint64_t* full_acc = empty_a + A_STAGES;
  uint64_t* empty_acc = full_acc + ACC_STAGES;
  uint64_t* drain = empty_acc + ACC_STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* prefix = reinterpret_cast<int*>(tmem_holder + 16);  // [E+1] m-tile prefix over experts

  const int warp = warp_id(), lane = lane_id();
  const int KB = (p.K + 63) / 64;
  const uint32_t sz_tx = p.sz_tma ? (uint32_t)(p.sz_rows * 128 * (p.s_es + p.z_es)) : 0u;

  if (threadIdx.x == 0) {
    for (int i = 0; i < X_STAGES; ++i) { mbar_init(&full_x[i], 1); mbar_init(&empty_x[i], 1); }
    for (int i = 0; i < W_STAGES; ++i) { mbar_init(&full_w[i], 1); mbar_init(&empty_w[i], 128); }
    for (int i = 0; i < A_STAGES; ++i) { mbar_init(&full_a[i], 128); mbar_init(&empty_a[i], 1); }
    for (int i = 0; i < ACC_STAGES; ++i) { mbar_init(&full_acc[i], 1); mbar_init(&empty_acc[i], 128); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    // m-tile prefix over the expert segments (dense: one segment of M rows), 32 experts per step
    int running = 0;
    for (int base = 0; base < p.E; base += 32) {
      const int e = base + lane;
      int v = 0;
      if (e < p.E) {
        const int cnt = p.offsets ? (p.offsets[e + 1] - p.offsets[e]) : p.M;
        v = (cnt + BT - 1) / BT;
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      if (e < p.E) prefix[e + 1] = running + v;
      running += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) prefix[0] = 0;
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmap_x);
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int num_tiles = prefix[p.E] * p.n_tiles_n;

  // tile -> (expert, first row, row end, n block)
  auto tile_info = [&](int tile, int& e, int& m0, int& mend, int& nb) {
    nb = tile % p.n_tiles_n;
    const int mt = tile / p.n_tiles_n;
    int lo = 0, hi = p.E;  // largest e with prefix[e] <= mt (skips empty experts)
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (prefix[mid] <= mt) lo = mid; else hi = mid;
    }
    e = lo;
    const int base = p.offsets ? p.offsets[e] : 0;
    m0 = base + (mt - prefix[e]) * BT;
    mend = p.offsets ? p.offsets[e + 1] : p.M;
  };

  if (warp == 0) {
    // activation tiles
    if (lane == 0) {
      int it = 0;
      int x_armed[X_STAGES];
      for (int i = 0; i < X_STAGES; ++i) x_armed[i] = -1;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int e, m0, mend, nb;
        tile_info(tile, e, m0, mend, nb);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int sx = it % X_STAGES, px = (it / X_STAGES) & 1;
          if (!mbar_wait(&empty_x[sx], px ^ 1, abort_flag, kDevErrTmaEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_x[sx], Cfg::kXStageBytes);
          const int kx = SWIGLU ? (kb < p.kb_x ? kb : kb - p.kb_x) : kb;  // gate half, then up half
          tma_load_2d(x_smem + sx * Cfg::kXStageBytes, &tmap_x, &full_x[sx], kx * 64, m0);
          x_armed[sx] = px;
        }
      }
      // every load issued lands before the CTA can exit (consumed ones return at once)
      for (int i = 0; i < X_STAGES; ++i)
        if (x_armed[i] >= 0) mbar_drain(&full_x[i], x_armed[i]);
    }
  } else if (warp == 2) {
    // packed weight tiles, decoupled from the activation stream
    if (lane == 0) {
      int it = 0;
      int w_armed[W_STAGES];
      for (int i = 0; i < W_STAGES; ++i) w_armed[i] = -1;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int e, m0, mend, nb;
        tile_info(tile, e, m0, mend, nb);
        const CUtensorMap* wm = p.wmaps + e;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int sw = it % W_STAGES, pw = (it / W_STAGES) & 1;
          if (!mbar_wait(&empty_w[sw], pw ^ 1, abort_flag, kDevErrWEmpty)) { ok = false; break; }
          uint8_t* ws = w_smem + sw * Cfg::kWStageBytes;
          mbar_arrive_expect_tx(&full_w[sw], Cfg::kWBytes + sz_tx);
          tma_load_2d(ws, wm, &full_w[sw], kb * Cfg::kKbBytes, nb * 128);
          if (p.sz_tma) {
            // the group rows of this 64-k block, [rows][128 features] each
            const int g0 = p.sz_rows > 1 ? kb * p.sz_rows : (kb * 64) / p.gs;
            tma_load_2d(ws + Cfg::kSOff, p.smaps + e, &full_w[sw], nb * 128, g0);
            tma_load_2d(ws + Cfg::kZOff, p.zmaps + e, &full_w[sw], nb * 128, g0);
          }
          w_armed[sw] = pw;
        }
      }
      // every load issued lands before the CTA can exit (consumed ones return at once)
      for (int i = 0; i < W_STAGES; ++i)
        if (w_armed[i] >= 0) mbar_drain(&full_w[i], w_armed[i]);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, tcount = 0;
      bool ok = true, issued = false;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++tcount) {
        // the MMA's N covers the tile's valid token rows (rounded up to 16): an expert segment
        // shorter than BT costs only its own rows of tensor-core time
        int e, m0, mend, nb;
        tile_info(tile, e, m0, mend, nb);
        const int valid = min(BT, mend - m0);
        const int n_mma = valid <= 0 ? 16 : min(BT, (valid + 15) & ~15);
        const uint32_t idesc = make_idesc_f16(BF16, 128, n_mma);
        // accumulator slots: one per tile, two in SwiGLU mode (gate, then up), taken in turn from a
        // ring of ACC_STAGES; a slot is free once the epilogue of its previous use has read it
        int slot = tcount * (SWIGLU ? 2 : 1);
        auto take = [&](int sl) {
          if (!mbar_wait(&empty_acc[sl % ACC_STAGES], ((sl / ACC_STAGES) & 1) ^ 1, abort_flag, kDevErrAccEmpty))
            return false;
          tc_fence_after();
          return true;
        };
        if (!take(slot)) { ok = false; break; }
        uint32_t d_tmem = tmem_base + (uint32_t)((slot % ACC_STAGES) * BT);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          // SwiGLU: the up half accumulates into the next slot, starting afresh
          const bool second = SWIGLU && kb >= p.kb_x;
          if (SWIGLU && kb == p.kb_x) {
            tc_commit(&full_acc[slot % ACC_STAGES]);  // the gate accumulator is complete
            ++slot;
            if (!take(slot)) { ok = false; break; }
            d_tmem = tmem_base + (uint32_t)((slot % ACC_STAGES) * BT);
          }
          const int kacc = second ? kb - p.kb_x : kb;
          const int sx = it % X_STAGES, px = (it / X_STAGES) & 1;
          const int sa = it % A_STAGES, pa = (it / A_STAGES) & 1;
          if (!mbar_wait(&full_x[sx], px, abort_flag, kDevErrTmaFull)) { ok = false; break; }
          if (!mbar_wait(&full_a[sa], pa, abort_flag, kDevErrAFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t xaddr = smem_u32(x_smem + sx * Cfg::kXStageBytes);
          const uint32_t a_tmem = tmem_base + (uint32_t)(Cfg::kAccCols + sa * 32);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tc_mma_ts(d_tmem, a_tmem + j * 8, smem_desc_kmajor_sw128(xaddr + j * 32), idesc, (kacc | j) != 0 ? 1u : 0u);
          issued = true;
          tc_commit(&empty_x[sx]);
          tc_commit(&empty_a[sa]);
        }
        if (!ok) break;
        tc_commit(&full_acc[slot % ACC_STAGES]);
      }
      if (!ok && issued) {
        tc_commit(drain);
        mbar_drain(drain, 0);
      }
    }
  } else if (warp >= 4 && warp < kRowsEpiWarp0) {
    // ------------------------------------------------------------ dequant warpgroups
    using Pp = Pair<BF16>;
    constexpr int kWords = Cfg::kKbBytes / 4;     // 32-bit words per row per k-block (8 or 4)
    constexpr int kSpan = 32 / WBITS;              // k per word (8 or 16)
    constexpr uint32_t kMask = WBITS == 4 ? 0x000F000Fu : 0x00030003u;
    const int wg = (warp - 4) >> 2;
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
      int e, m0, mend, nb;
      tile_info(tile, e, m0, mend, nb);
      const int n = nb * 128 + row;
      const int nn = n < p.N ? n : 0;
      const void* sb = p.sptr[e];
      const void* zb = p.zptr[e];
      const long long s_row = (long long)nn * p.s_stride_n;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        if ((it % kRowsDqGroups) != wg) continue;
        const int sw = it % W_STAGES, pw = (it / W_STAGES) & 1;
        const int sa = it % A_STAGES, pa = (it / A_STAGES) & 1;
        // group of each word of the block: one division per k-block, then the group advances
        // where a word starts on a group boundary (gs is a multiple of kSpan)
        const int kbase = kb * 64;
        const uint8_t* st = w_smem + sw * Cfg::kWStageBytes;
        // scale and zero of word w (group grp): from the stage (staged by TMA, [rows][128]) or global
        auto fetch = [&](int w, int grp, float& sv, float& zv) {
          if (p.sz_tma) {
            const int slot = p.sz_rows > 1 ? (w * kSpan) / p.gs : 0;
            sv = load_as_f32(st + Cfg::kSOff, p.s_dtype, slot * 128 + row);
            zv = load_as_f32(st + Cfg::kZOff, p.z_dtype, slot * 128 + row);
          } else {
            const long long si = s_row + (long long)grp * p.s_stride_g;
            sv = load_as_f32(sb, p.s_dtype, si);
            zv = load_as_f32(zb, p.z_dtype, si);
          }
        };
        uint32_t r32[32];
        uint32_t q[kWords];
        auto load_q = [&]() {
          const uint32_t* wt = reinterpret_cast<const uint32_t*>(st + row * Cfg::kKbBytes);
#pragma unroll
          for (int w = 0; w < kWords; w += 4) {
            const uint4 v = *reinterpret_cast<const uint4*>(wt + w);
            q[w] = v.x; q[w + 1] = v.y; q[w + 2] = v.z; q[w + 3] = v.w;
          }
        };
        if constexpr (MODE == kRowsExact && WBITS == 2) {
          // Table decode, bit-exact for any scale and zero: per (row, group) the four weights
          // RNE((c - z) * s), c = 0..3, are computed in fp32 as the reference does and rounded
          // once; their low bytes form tlo and their high bytes thi, so a code c selects byte c
          // of each, and one prmt per table turns four codes into their four values' bytes.
          uint32_t tlo[kWords], thi[kWords];
          auto build = [&]() {
            int grp = kbase / p.gs;
            int next_k = (grp + 1) * p.gs;
#pragma unroll
            for (int w = 0; w < kWords; ++w) {
              const int k0 = kbase + w * kSpan;
              const bool fresh = (w == 0) || (k0 >= next_k && k0 < p.K);
              if (w > 0 && fresh) {
                ++grp;
                next_k += p.gs;
              }
              if (fresh) {
                float sv, zv;
                fetch(w, k0 < p.K ? grp : 0, sv, zv);
                const uint32_t p01 = pack2_rn<BF16>(__fmul_rn(__fsub_rn(0.f, zv), sv), __fmul_rn(__fsub_rn(1.f, zv), sv));
                const uint32_t p23 =
                    pack2_rn<BF16>(__fmul_rn(__fsub_rn(2.f, zv), sv), __fmul_rn(__fsub_rn(3.f, zv), sv));
                tlo[w] = prmt(p01, p23, 0x6420u);
                thi[w] = prmt(p01, p23, 0x7531u);
              } else {
                tlo[w] = tlo[w > 0 ? w - 1 : 0];
                thi[w] = thi[w > 0 ? w - 1 : 0];
              }
            }
          };
          if (!p.sz_tma) build();  // global loads in flight while the weight stage lands
          if (!mbar_wait(&full_w[sw], pw, abort_flag, kDevErrWFull)) { ok = false; break; }
          if (p.sz_tma) build();
          load_q();
          mbar_arrive(&empty_w[sw]);
#pragma unroll
          for (int w = 0; w < kWords; ++w) {
            // nibble i of u holds code 2i, nibble i of v code 2i + 1; x gathers codes
            // (4b, 4b+2, 4b+1, 4b+3) as four byte selectors
            const uint32_t u = q[w] & 0x33333333u, v = (q[w] >> 2) & 0x33333333u;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const uint32_t x = prmt(u, v, 0x40u + 0x11u * (uint32_t)b);
              const uint32_t lo = prmt(tlo[w], tlo[w], x), hi = prmt(thi[w], thi[w], x);
              r32[8 * w + 2 * b] = prmt(lo, hi, 0x6240u);      // codes 4b, 4b+1
              r32[8 * w + 2 * b + 1] = prmt(lo, hi, 0x7351u);  // codes 4b+2, 4b+3
            }
          }
        } else {
          RowsConst<BF16, MODE> cst[kWords];
          bool exact = true;  // exact mode: the pair arithmetic reproduces the fp32 formula
          auto build = [&]() {
            int grp = kbase / p.gs;
            int next_k = (grp + 1) * p.gs;
#pragma unroll
            for (int w = 0; w < kWords; ++w) {
              const int k0 = kbase + w * kSpan;
              const bool fresh = (w == 0) || (k0 >= next_k && k0 < p.K);
              if (w > 0 && fresh) {
                ++grp;
                next_k += p.gs;
              }
              if (fresh) {
                float sv, zv;
                fetch(w, k0 < p.K ? grp : 0, sv, zv);
                cst[w] = rows_const<BF16, MODE>(sv, zv);
                if (MODE == kRowsExact) exact = exact && rows_pair_exact<BF16, MODE>(sv, zv, cst[w]);
              } else {
                cst[w] = cst[w > 0 ? w - 1 : 0];
              }
            }
          };
          if (!p.sz_tma) build();
          if (!mbar_wait(&full_w[sw], pw, abort_flag, kDevErrWFull)) { ok = false; break; }
          if (p.sz_tma) build();
          load_q();
          if (MODE == kRowsRtn || __all_sync(0xffffffffu, exact)) {
            mbar_arrive(&empty_w[sw]);
#pragma unroll
            for (int w = 0; w < kWords; ++w) {
              const uint32_t qq = q[w];
              const uint32_t p0 = rows_dq<BF16, MODE, HAS_LO>(lop3_and_or(qq, kMask, Pp::kMagic), cst[w]);
              const uint32_t p1 = rows_dq<BF16, MODE, HAS_LO>(lop3_and_or(qq >> 4, kMask, Pp::kMagic), cst[w]);
              const uint32_t p2 = rows_dq<BF16, MODE, HAS_LO>(lop3_and_or(qq >> 8, kMask, Pp::kMagic), cst[w]);
              const uint32_t p3 = rows_dq<BF16, MODE, HAS_LO>(lop3_and_or(qq >> 12, kMask, Pp::kMagic), cst[w]);
              r32[4 * w + 0] = prmt(p0, p1, 0x5410u);
              r32[4 * w + 1] = prmt(p2, p3, 0x5410u);
              r32[4 * w + 2] = prmt(p0, p1, 0x7632u);
              r32[4 * w + 3] = prmt(p2, p3, 0x7632u);
            }
          } else {
            // zeros or scales the pair arithmetic cannot reproduce exactly (a zero that is not a
            // half-integer, an fp32 scale, a scale outside the pair type's range): the reference's
            // formula in fp32, RNE((q - z) * s), for every weight of the warp's block (the stage is
            // released after this decode: the staged scales are read here again)
#pragma unroll
            for (int w = 0; w < kWords; ++w) {
              const int k0 = kbase + w * kSpan;
              float sv, zv;
              fetch(w, k0 < p.K ? k0 / p.gs : 0, sv, zv);
              const uint32_t qq = q[w];
#pragma unroll
              for (int j = 0; j < 8; j += 2) {
                const float qa = (float)((qq >> (4 * j)) & 0xFu), qb = (float)((qq >> (4 * j + 4)) & 0xFu);
                r32[4 * w + j / 2] =
                    pack2_rn<BF16>(__fmul_rn(__fsub_rn(qa, zv), sv), __fmul_rn(__fsub_rn(qb, zv), sv));
              }
            }
            mbar_arrive(&empty_w[sw]);
          }
        }
        if (!mbar_wait(&empty_a[sa], pa ^ 1, abort_flag, kDevErrAEmpty)) { ok = false; break; }
        tc_fence_after();
        __syncwarp();
        const uint32_t taddr = tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(Cfg::kAccCols + sa * 32);
        tmem_st_32x32b_x32(taddr, r32);
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&full_a[sa]);
      }
    }
  } else if (warp >= kRowsEpiWarp0) {
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const int odt = BF16 ? kBF16 : kF16;
    int tcount = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tcount) {
      const int s0 = tcount * (SWIGLU ? 2 : 1);                 // this tile's first accumulator slot
      const int sc = s0 % ACC_STAGES, pc = (s0 / ACC_STAGES) & 1;
      const int su = (s0 + 1) % ACC_STAGES, pu = ((s0 + 1) / ACC_STAGES) & 1;   // SwiGLU: the up slot
      int e, m0, mend, nb;
      tile_info(tile, e, m0, mend, nb);
      const int n = nb * 128 + row;
      const bool nvalid = n < p.N;
      const float bv = (p.bias && nvalid) ? load_as_f32(p.bias, p.bias_dtype, n) : 0.f;
      if (!mbar_wait(&full_acc[sc], pc, abort_flag, kDevErrAccFull)) break;
      if (SWIGLU && !mbar_wait(&full_acc[su], pu, abort_flag, kDevErrAccFull)) break;
      tc_fence_after();
      __syncwarp();
      const uint32_t tbase = tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(sc * BT);
      const uint32_t ubase = tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(su * BT);
      if constexpr (SWIGLU) {
        // 16 token rows at a time (BT is a multiple of 16): the gate and up values of 32 rows at
        // once would not fit the registers
        const int n16 = min(BT / 16, (mend - m0 + 15) / 16);
#pragma unroll 1
        for (int c = 0; c < n16; ++c) {
          uint32_t gq[16], uq[16];
          tmem_ld_32x32b_x16(tbase + (uint32_t)(c * 16), gq);
          tmem_ld_32x32b_x16(ubase + (uint32_t)(c * 16), uq);
          tc_wait_ld();
          if (nvalid) {
            const int rh = m0 + 16 * c;
            uint16_t* dst = p.out + (long long)rh * p.ldc + n;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (rh + i < mend) {
                // the gate and up outputs as their own GEMMs would store them, then silu(g) * u
                const float gv = bits_to_f32(f32_to_bits(__uint_as_float(gq[i]) + bv, odt), odt);
                const float uv = bits_to_f32(f32_to_bits(__uint_as_float(uq[i]) + bv, odt), odt);
                dst[(long long)i * p.ldc] = f32_to_bits(silu_f32(gv) * uv, odt);
              }
          }
        }
        tc_fence_before();
        mbar_arrive(&empty_acc[sc]);
        mbar_arrive(&empty_acc[su]);
        continue;
      }
      const int nch = min(BT / 32, (mend - m0 + 31) / 32);  // chunks holding valid rows
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const int r0 = m0 + c * 32;
        uint32_t v[32];
        tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), v);
        tc_wait_ld();
        if (nvalid) {
          uint16_t* dst = p.out + (long long)r0 * p.ldc + n;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (r0 + i < mend) dst[(long long)i * p.ldc] = f32_to_bits(__uint_as_float(v[i]) + bv, odt);
        }
      }
      tc_fence_before();
      mbar_arrive(&empty_acc[sc]);
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
