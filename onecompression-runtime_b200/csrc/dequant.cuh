// Standalone unpack / dequant / repack kernels.
//
// All dequant kernels reproduce the reference's rounding exactly:
//  * GPTQ  (quant_utils.py:50-69)          w = RNE_out( f32(s) * (f32(q) - f32(z)) )  -- one rounding
//  * RTN   (quant_utils.py:72-103)         d = RNE_out(q - RNE_out(z)); w = RNE_out(d * RNE_out(s))
//                                          (fp32 output: w = f32(f32(q - z) * s))
//  * DSV4  (dsv4_packed_linear.py:22-56)   w = RNE_out( f32(f32(q) - z) * s )      -- fp32 ops, one cast
#pragma once

#include "common.cuh"

namespace oc {

// --- GPTQ dequant: qweight [K/pf, N] int32 -> W [N, K] (nn.Linear layout) -------------
// Block: 32 (n) x 8 (word rows). Each thread expands one word; the tile is
// transposed through shared memory so the [N, K] rows are written with
// coalesced 16-byte stores.
template <int WBITS>
__global__ void __launch_bounds__(256) gptq_dequant_kernel(const uint32_t* __restrict__ qw,
                                                           const uint32_t* __restrict__ qz,
                                                           const void* __restrict__ scales, int s_dtype,
                                                           const long long* __restrict__ g_idx, int K, int N,
                                                           int G, int gs, int v1, uint16_t* __restrict__ out,
                                                           int out_dtype) {
  constexpr int PF = 32 / WBITS;         // values per word
  constexpr uint32_t MASK = (1u << WBITS) - 1u;
  __shared__ uint16_t tile[32][8 * PF + 2];  // [n][k within tile]
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int n0 = blockIdx.x * 32, kw0 = blockIdx.y * 8;
  const int n = n0 + tx, kw = kw0 + ty;
  const int kw_rows = (K + PF - 1) / PF;
  if (n < N && kw < kw_rows) {
    const uint32_t word = qw[(long long)kw * N + n];
#pragma unroll
    for (int i = 0; i < PF; ++i) {
      const int k = kw * PF + i;
      uint16_t v = 0;
      if (k < K) {
        const long long g = g_idx ? g_idx[k] : (long long)(k / gs);
        const uint32_t zw = qz[g * (long long)(N / PF) + n / PF];
        uint32_t z = (zw >> (WBITS * (n % PF))) & MASK;
        if (v1) z = (z + 1u) & MASK;
        const float s = load_as_f32(scales, s_dtype, g * (long long)N + n);
        const uint32_t q = (word >> (WBITS * i)) & MASK;
        const float prod = __fmul_rn(s, __fsub_rn((float)q, (float)z));
        v = f32_to_bits(prod, out_dtype);
      }
      tile[tx][ty * PF + i] = v;
    }
  }
  __syncthreads();
  // write: each of the 32 rows has 8*PF values; threads take 2-value chunks
  const int kbase = kw0 * PF;
  for (int idx = threadIdx.x; idx < 32 * 4 * PF; idx += 256) {
    const int r = idx / (4 * PF), c = (idx % (4 * PF)) * 2;
    const int nn = n0 + r, k = kbase + c;
    if (nn < N && k < K) {
      uint16_t* dst = out + (long long)nn * K + k;
      if (k + 1 < K && ((reinterpret_cast<uintptr_t>(dst) & 3u) == 0)) {
        *reinterpret_cast<uint32_t*>(dst) = pack2(tile[r][c], tile[r][c + 1]);
      } else {
        dst[0] = tile[r][c];
        if (k + 1 < K) dst[1] = tile[r][c + 1];
      }
    }
  }
}

// fp32 output (dequant_gptq_to_fp with dtype=float32): the fp32 product itself.
__global__ void gptq_dequant_f32_kernel(const uint32_t* __restrict__ qw, const uint32_t* __restrict__ qz,
                                        const void* __restrict__ scales, int s_dtype,
                                        const long long* __restrict__ g_idx, int K, int N, int gs, int wbits, int v1,
                                        float* __restrict__ out) {
  const int pf = 32 / wbits;
  const uint32_t mask = (1u << wbits) - 1u;
  const long long total = (long long)N * K;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / K), k = (int)(i % K);
    const long long g = g_idx ? g_idx[k] : (long long)(k / gs);
    uint32_t z = (qz[g * (long long)(N / pf) + n / pf] >> (wbits * (n % pf))) & mask;
    if (v1) z = (z + 1u) & mask;
    const uint32_t q = (qw[(long long)(k / pf) * N + n] >> (wbits * (k % pf))) & mask;
    out[i] = __fmul_rn(load_as_f32(scales, s_dtype, g * (long long)N + n), __fsub_rn((float)q, (float)z));
  }
}

// --- GPTQ unpack (a1): qweight -> int [N, K]; qzeros -> int [G, N] ----------------------
__global__ void gptq_unpack_kernel(const uint32_t* __restrict__ qw, int K, int N, int wbits,
                                   int32_t* __restrict__ out) {
  const long long total = (long long)K * N;
  const int pf = 32 / wbits;
  const uint32_t mask = (1u << wbits) - 1u;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / K), k = (int)(i % K);
    const uint32_t w = qw[(long long)(k / pf) * N + n];
    out[i] = (int32_t)((w >> (wbits * (k % pf))) & mask);
  }
}

__global__ void gptq_unpack_zeros_kernel(const uint32_t* __restrict__ qz, int G, int N, int wbits,
                                         int32_t* __restrict__ out) {
  const long long total = (long long)G * N;
  const int pf = 32 / wbits;
  const uint32_t mask = (1u << wbits) - 1u;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(i / N), n = (int)(i % N);
    const uint32_t w = qz[(long long)g * (N / pf) + n / pf];
    out[i] = (int32_t)((w >> (wbits * (n % pf))) & mask);
  }
}

// --- GPTQ pack (a3): int [N, K] -> qweight [K/pf, N] ------------------------------------
__global__ void gptq_pack_kernel(const int32_t* __restrict__ w, int N, int K, int wbits,
                                 uint32_t* __restrict__ qw) {
  const int pf = 32 / wbits;
  const int rows = (K + pf - 1) / pf;
  const long long total = (long long)rows * N;
  const uint32_t mask = (1u << wbits) - 1u;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / N), n = (int)(i % N);
    uint32_t acc = 0;
    for (int j = 0; j < pf; ++j) {
      const int k = r * pf + j;
      if (k < K) acc |= ((uint32_t)w[(long long)n * K + k] & mask) << (wbits * j);
    }
    qw[i] = acc;
  }
}

// --- K re-layout for act-order / odd groups: qw'[w', n] = pack_i q(kperm[8w'+i], n) ------
// kperm[k'] = source k, or -1 for a padding row (code 0).
__global__ void gptq_repack_k_kernel(const uint32_t* __restrict__ qw, const int32_t* __restrict__ kperm,
                                     int Kp, int N, uint32_t* __restrict__ out) {
  const int rows = Kp / 8;
  const long long total = (long long)rows * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / N), n = (int)(i % N);
    uint32_t acc = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int src = kperm[r * 8 + j];
      if (src >= 0) {
        const uint32_t w = qw[(long long)(src >> 3) * N + n];
        acc |= ((w >> (4 * (src & 7))) & 0xFu) << (4 * j);
      }
    }
    out[i] = acc;
  }
}

// 8-bit codes (4 per word): qweight_out[w', n] packs, for i < 4, the code of source row
// kperm[4w'+i] (0 when it is -1).
__global__ void gptq_repack_k8_kernel(const uint32_t* __restrict__ qw, const int32_t* __restrict__ kperm,
                                      int Kp, int N, uint32_t* __restrict__ out) {
  const long long total = (long long)(Kp / 4) * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / N), n = (int)(i % N);
    uint32_t acc = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int src = kperm[r * 4 + j];
      if (src >= 0) acc |= ((qw[(long long)(src >> 2) * N + n] >> (8 * (src & 3))) & 0xFFu) << (8 * j);
    }
    out[i] = acc;
  }
}

// --- activation gather: x'[m, k'] = x[m, kperm[k']] (0 for -1) --------------------------
__global__ void permute_cols_kernel(const uint16_t* __restrict__ x, long long ldx, int M, int K,
                                    const int32_t* __restrict__ kperm, int Kp, uint16_t* __restrict__ out) {
  // Launched with programmatic stream serialization: let the next kernel (the GEMV, which
  // prefetches its weights meanwhile) launch, and wait for the kernel that produced x.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const long long total = (long long)M * Kp;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / Kp), kp = (int)(i % Kp);
    const int src = kperm[kp];
    out[i] = (src >= 0 && src < K) ? x[(long long)m * ldx + src] : (uint16_t)0;
  }
}

// --- im2col of a 1-D convolution input: the A operand of Conv1d run as a GEMM ----------
// a[(b T + t) lda + c ksize + k] = x[b, c, t stride + k dil - pad] (0 outside [0, L)), for
// columns < C ksize; columns up to cols_out are written as 0 (the GEMM's zero-padded K). x element
// (b, c, l) sits at b sxb + c sxc + l (16-bit values). Writes are coalesced along the columns.
__global__ void im2col1d_kernel(const uint16_t* __restrict__ x, long long sxb, long long sxc, int C, int L,
                                int ksize, int stride, int dil, int pad, int T, int cols_out, long long rows,
                                uint16_t* __restrict__ a, long long lda) {
  const int ck_total = C * ksize;
  const long long total = rows * cols_out;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int col = (int)(i % cols_out);
    const long long bt = i / cols_out;
    uint16_t v = 0;
    if (col < ck_total) {
      const int t = (int)(bt % T);
      const long long b = bt / T;
      const int c = col / ksize, k = col - c * ksize;
      const int l = t * stride + k * dil - pad;
      if (l >= 0 && l < L) v = x[b * sxb + (long long)c * sxc + l];
    }
    a[bt * lda + col] = v;
  }
}

// --- RTN uint8-nibble dequant (a11) ----------------------------------------------------
// One element of torch's (q.to(dt) - z.to(dt)) * s.to(dt): for 16-bit dt a rounding after
// each cast and op; for fp32 the casts are exact and each op rounds once.
__device__ __forceinline__ void rtn_store(void* out, long long i, float qv, float zv, float sv, int out_dtype) {
  if (out_dtype == kF32) {
    static_cast<float*>(out)[i] = __fmul_rn(__fsub_rn(qv, zv), sv);
    return;
  }
  const float zo = bits_to_f32(f32_to_bits(zv, out_dtype), out_dtype);
  const float so = bits_to_f32(f32_to_bits(sv, out_dtype), out_dtype);
  const float d = bits_to_f32(f32_to_bits(__fsub_rn(qv, zo), out_dtype), out_dtype);
  static_cast<uint16_t*>(out)[i] = f32_to_bits(__fmul_rn(d, so), out_dtype);
}

// qweight_u8 [N, ldq] bytes: low nibble = even k. scales/zeros [N, G] (f16/bf16/f32);
// output f16, bf16 or f32.
__global__ void rtn_dequant_kernel(const uint8_t* __restrict__ q, long long ldq, const void* __restrict__ s,
                                   int s_dtype, const void* __restrict__ z, int z_dtype, int K, int N, int G,
                                   void* __restrict__ out, int out_dtype) {
  const long long total = (long long)N * K;
  const int gs = K / G;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / K), k = (int)(i % K);
    const uint8_t b = q[(long long)n * ldq + (k >> 1)];
    const float qv = (float)((k & 1) ? (b >> 4) : (b & 0xF));
    const int g = (G == 1) ? 0 : (k / gs);
    const long long si = (long long)n * G + g;
    rtn_store(out, i, qv, load_as_f32(z, z_dtype, si), load_as_f32(s, s_dtype, si), out_dtype);
  }
}

// --- RTN packed embedding: gather + dequant ------------------------------------------
// out[i, k] = dequant of row ids[i] of the table (same arithmetic as rtn_dequant_kernel).
// Negative ids count from the end of the table, as torch indexing does; an id outside
// [-vocab, vocab) records kDevErrIndex and yields a zero row (no out-of-bounds read).
__global__ void rtn_embedding_kernel(const int64_t* __restrict__ ids, long long n_ids, long long vocab,
                                     const uint8_t* __restrict__ q, long long ldq, const void* __restrict__ s,
                                     int s_dtype, const void* __restrict__ z, int z_dtype, int K, int G,
                                     void* __restrict__ out, int out_dtype) {
  const long long total = n_ids * K;
  const int gs = K / G;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / K;
    const int k = (int)(i % K);
    long long n = ids[r];
    if (n < 0) n += vocab;
    if (n < 0 || n >= vocab) {
      if (k == 0) record_error(kDevErrIndex);
      if (out_dtype == kF32) static_cast<float*>(out)[i] = 0.f;
      else static_cast<uint16_t*>(out)[i] = 0;
      continue;
    }
    const uint8_t b = q[n * ldq + (k >> 1)];
    const float qv = (float)((k & 1) ? (b >> 4) : (b & 0xF));
    const int g = (G == 1) ? 0 : (k / gs);
    rtn_store(out, i, qv, load_as_f32(z, z_dtype, n * G + g), load_as_f32(s, s_dtype, n * G + g), out_dtype);
  }
}

// --- DSV4 int4/int2 dequant (a12) ------------------------------------------------------
// packed [N, ldq] bytes, code j of a byte at bits j*wbits. scales/zeros indexed
// through (s_row_stride, s_col_stride) so both [N, G] and [G, N] layouts work.
__global__ void dsv4_dequant_kernel(const uint8_t* __restrict__ q, long long ldq, int wbits,
                                    const void* __restrict__ s, int s_dtype, const void* __restrict__ z,
                                    int z_dtype, long long s_stride_n, long long s_stride_g, int gs, int K,
                                    int N, uint16_t* __restrict__ out, int out_dtype) {
  const long long total = (long long)N * K;
  const int per = 8 / wbits;
  const uint32_t mask = (1u << wbits) - 1u;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / K), k = (int)(i % K);
    const uint8_t b = q[(long long)n * ldq + k / per];
    const float qv = (float)((b >> (wbits * (k % per))) & mask);
    const int g = gs > 0 ? k / gs : 0;
    const long long si = (long long)n * s_stride_n + (long long)g * s_stride_g;
    const float sv = load_as_f32(s, s_dtype, si);
    const float zv = load_as_f32(z, z_dtype, si);
    out[i] = f32_to_bits(__fmul_rn(__fsub_rn(qv, zv), sv), out_dtype);
  }
}

}  // namespace oc
