// to_fp8 on the GPU: per-tensor amax -> scale, and the e4m3 quantiser
// (lib_sparse/fp8.py:123-129), in either of two arithmetics: eager
// PyTorch's for a bf16 / fp32 tensor (scale = max(amax / 448, 1e-9) with the
// quotient rounded to the input dtype, q = e4m3(x / scale) with the quotient
// rounded to the input dtype first), or -- `compiled` -- that of the
// reference's @torch.compile'd to_fp8 on a GPU (scale = max(amax * (1/448),
// 1e-9) in fp32, q = e4m3(x / scale) with Triton's fp32 division).
#include "common.cuh"

namespace bs {

// ---------------------------------------------------------------------------
// to_fp8 scale: amax(|x|) -> scale (lib_sparse/fp8.py:123-129)
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(kThreads)
amax_kernel(const uint8_t *x, int64_t n, uint32_t *amax_ws) {
  constexpr int EB = Elt<DT>::bytes;
  const int64_t nvec = (n * EB) / 16;
  float m = 0.f;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nvec; i += stride) {
    const uint4 v = ld_nc_v4(x + 16 * i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if constexpr (DT == BS_BF16) {
        m = fmaxf(m, fabsf(bf16_bits_to_f32(w[q] & 0xFFFFu)));
        m = fmaxf(m, fabsf(bf16_bits_to_f32(w[q] >> 16)));
      } else {
        m = fmaxf(m, fabsf(__uint_as_float(w[q])));
      }
    }
  }
  // scalar tail
  for (int64_t e = nvec * (16 / EB) + (int64_t)blockIdx.x * kThreads + threadIdx.x; e < n;
       e += stride) {
    if constexpr (DT == BS_BF16)
      m = fmaxf(m, fabsf(bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(x)[e])));
    else
      m = fmaxf(m, fabsf(reinterpret_cast<const float *>(x)[e]));
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, d));
  __shared__ float s_m[kThreads / 32];
  if ((threadIdx.x & 31) == 0) s_m[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.f;
    for (int i = 0; i < kThreads / 32; ++i) b = fmaxf(b, s_m[i]);
    atomicMax(amax_ws, __float_as_uint(b));  // non-negative floats order as uints
  }
}

// Finalise the scale and reset the scratch word for the next call.
template <int DT>
__global__ void scale_kernel(uint32_t *amax_ws, float *scale_out, int compiled) {
  const float amax = __uint_as_float(*amax_ws);
  // eager divides by 448; the compiled function multiplies by 1/448 rounded
  // to fp32 (Inductor's rewrite of a division by a constant)
  float s = compiled ? amax * kRcp448 : __fdiv_rn(amax, 448.0f);
  if (DT == BS_BF16 && !compiled) s = bf16_bits_to_f32(f32_to_bf16_bits(s));
  *scale_out = fmaxf(s, 1e-9f);  // clamp(min=1e-9)
  *amax_ws = 0u;
}

// amax of h = relu(bf16(z + bias)) over a bf16 [M, N] tensor (row stride
// ld), the input of to_fp8 in the fused FFN forward: bias add and ReLU as
// torch computes them, no h materialised.
__global__ void __launch_bounds__(kThreads)
amax_bias_relu_kernel(const uint8_t *z, int64_t M, int64_t N, int64_t ld, const uint8_t *bias,
                      uint32_t *amax_ws) {
  const int64_t cpr = (N + 7) / 8;  // 8-column chunks per row
  const bool vec = (N % 8 == 0) && (ld % 8 == 0);
  float m = 0.f;
  // a block walks rows blockIdx.x, + gridDim.x, ... chunk by chunk, its
  // threads kThreads chunks apart: one division per thread, not per chunk
  const int64_t dr = kThreads / cpr, di = kThreads % cpr;
  for (int64_t i = threadIdx.x % cpr, r = blockIdx.x + (threadIdx.x / cpr) * gridDim.x; r < M;) {
    const int64_t c0 = i * 8;
    uint32_t zw[4] = {0, 0, 0, 0}, bw[4] = {0, 0, 0, 0};
    if (vec) {
      const uint4 v = ld_nc_v4(z + (r * ld + c0) * 2);
      const uint4 b = *reinterpret_cast<const uint4 *>(bias + c0 * 2);
      zw[0] = v.x; zw[1] = v.y; zw[2] = v.z; zw[3] = v.w;
      bw[0] = b.x; bw[1] = b.y; bw[2] = b.z; bw[3] = b.w;
    } else {
      for (int e = 0; e < 8 && c0 + e < N; ++e) {
        zw[e >> 1] |= (uint32_t)reinterpret_cast<const uint16_t *>(z)[r * ld + c0 + e] << (16 * (e & 1));
        bw[e >> 1] |= (uint32_t)reinterpret_cast<const uint16_t *>(bias)[c0 + e] << (16 * (e & 1));
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = bf16_bits_to_f32(zw[q] & 0xFFFFu) + bf16_bits_to_f32(bw[q] & 0xFFFFu);
      const float hi = bf16_bits_to_f32(zw[q] >> 16) + bf16_bits_to_f32(bw[q] >> 16);
      const uint32_t h = relu_bf16x2(bf16x2_from_f32(lo, hi));
      m = fmaxf(m, fabsf(bf16_bits_to_f32(h & 0xFFFFu)));
      m = fmaxf(m, fabsf(bf16_bits_to_f32(h >> 16)));
    }
    i += di;
    r += dr * gridDim.x;
    if (i >= cpr) {
      i -= cpr;
      r += gridDim.x;
    }
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, d));
  __shared__ float s_m[kThreads / 32];
  if ((threadIdx.x & 31) == 0) s_m[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.f;
    for (int i = 0; i < kThreads / 32; ++i) b = fmaxf(b, s_m[i]);
    atomicMax(amax_ws, __float_as_uint(b));  // non-negative floats order as uints
  }
}

// The to_fp8 scales of h (bf16) and of h2 = bf16(h * h) from amax(h): h2 is
// a non-decreasing function of h >= 0 and rounding is monotonic, so
// amax(h2) = bf16(amax(h)^2) exactly; both scales follow scale_kernel's
// bf16 rule.  Resets the scratch word.
__global__ void scales_relu2_kernel(uint32_t *amax_ws, float *scale_h, float *scale_h2,
                                    int compiled) {
  const float amax = __uint_as_float(*amax_ws);
  float s = compiled ? amax * kRcp448 : __fdiv_rn(amax, 448.0f);
  if (!compiled) s = bf16_bits_to_f32(f32_to_bf16_bits(s));
  *scale_h = fmaxf(s, 1e-9f);
  if (scale_h2) {
    const float a2 = bf16_bits_to_f32(f32_to_bf16_bits(amax * amax));
    s = compiled ? a2 * kRcp448 : __fdiv_rn(a2, 448.0f);
    if (!compiled) s = bf16_bits_to_f32(f32_to_bf16_bits(s));
    *scale_h2 = fmaxf(s, 1e-9f);
  }
  *amax_ws = 0u;
}

// q = e4m3(x / scale) over a flat tensor (the quantise half of to_fp8).
template <int DT>
__global__ void __launch_bounds__(kThreads)
quant_kernel(const uint8_t *x, int64_t n, const float *scale, uint8_t *q, int compiled) {
  const float s = *scale;
  const float r = quant_rcp(s);
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  // with 16+ groups per thread the once-per-block exactness check of the
  // plain estimate pays for itself (the condition is uniform over the grid)
  bool fast = false;
  if constexpr (DT == BS_BF16)
    if ((n + 7) / 8 >= 16 * stride) fast = e4m3_estimate_exact(s, r, compiled != 0);
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i * 8 < n; i += stride) {
    uint32_t o[2] = {0, 0};
    const int64_t e0 = i * 8;
    const bool full = e0 + 8 <= n;
    uint32_t b[8];
    if constexpr (DT == BS_BF16) {
      if (full) {
        const uint4 v = ld_nc_v4(x + e0 * 2);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) b[e] = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
      } else {
        for (int e = 0; e < 8; ++e)
          b[e] = e0 + e < n ? reinterpret_cast<const uint16_t *>(x)[e0 + e] : 0u;
      }
    } else {
      if (full) {
        const uint4 v0 = ld_nc_v4(x + e0 * 4), v1 = ld_nc_v4(x + e0 * 4 + 16);
        b[0] = v0.x; b[1] = v0.y; b[2] = v0.z; b[3] = v0.w;
        b[4] = v1.x; b[5] = v1.y; b[6] = v1.z; b[7] = v1.w;
      } else {
        for (int e = 0; e < 8; ++e)
          b[e] = e0 + e < n ? reinterpret_cast<const uint32_t *>(x)[e0 + e] : 0u;
      }
    }
    if constexpr (DT == BS_BF16) {
      // |x / scale| <= 448 * (1 + 2^-8) by construction of the scale, so the
      // fast e4m3 conversion applies (NaN stays NaN).
      const uint32_t w4[4] = {b[0] | b[1] << 16, b[2] | b[3] << 16, b[4] | b[5] << 16,
                              b[6] | b[7] << 16};
      if (fast) {
        if (compiled) est_e4m3x8<true>(w4, r, o);
        else est_e4m3x8<false>(w4, r, o);
      } else if (compiled) {
        full_e4m3x8(w4, s, r, o);
      } else {
        div_e4m3x8(w4, s, r, o);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (compiled) {
          o[e >> 2] |= e4m3_compiled(__uint_as_float(b[e]), s, r) << (8 * (e & 3));
          continue;
        }
        const float y = __fdiv_rn(__uint_as_float(b[e]), s);
        o[e >> 2] |= f32_to_e4m3_bits(y) << (8 * (e & 3));
      }
    }
    if (full) {
      *reinterpret_cast<uint2 *>(q + e0) = make_uint2(o[0], o[1]);
    } else {
      for (int e = 0; e < 8 && e0 + e < n; ++e) q[e0 + e] = (o[e >> 2] >> (8 * (e & 3))) & 0xFFu;
    }
  }
}

// to_fp8's quantiser on a bf16 [R, C] tensor (row stride ld) into either or
// both fp8 layouts: q [R, C] (row stride ldq) and qT [C, R] (row stride
// ldqT), the transposed copy cuBLASLt's fp8 GEMMs want for an operand in the
// other major order -- one read of the bf16 tensor instead of a quantise
// pass plus a transpose pass over its fp8 copy.  A CTA quantises a 64 x 64
// tile (16 values per thread, div_e4m3x8) and, for qT, turns it through
// shared memory.
__global__ void __launch_bounds__(kThreads)
quant2d_kernel(const uint8_t *x, int64_t R, int64_t C, int64_t ld, const float *scale,
               uint8_t *q, int64_t ldq, uint8_t *qT, int64_t ldqT, int vx, int vq, int vqT,
               int compiled) {
  __shared__ uint8_t t[64][64 + 4];
  const float s = *scale;
  const float rc = quant_rcp(s);
  const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
  const int tid = threadIdx.x;
  {  // row tid/4, 16 values at column (tid%4)*16
    const int r = tid >> 2, cq = (tid & 3) * 16;
    const int64_t gr = r0 + r, gc = c0 + cq;
    uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const bool full = gr < R && gc + 16 <= C;
    if (gr < R) {
      const uint8_t *src = x + (gr * ld + gc) * 2;
      if (vx && full) {
        const uint4 v0 = ld_nc_v4(src), v1 = ld_nc_v4(src + 16);
        w[0] = v0.x; w[1] = v0.y; w[2] = v0.z; w[3] = v0.w;
        w[4] = v1.x; w[5] = v1.y; w[6] = v1.z; w[7] = v1.w;
      } else {
        for (int e = 0; e < 16; ++e)
          if (gc + e < C)
            w[e >> 1] |= (uint32_t)reinterpret_cast<const uint16_t *>(src)[e] << (16 * (e & 1));
      }
    }
    uint32_t o[4];
    {
      const uint32_t lo[4] = {w[0], w[1], w[2], w[3]}, hi[4] = {w[4], w[5], w[6], w[7]};
      uint32_t o2[2];
      if (compiled) full_e4m3x8(lo, s, rc, o2);
      else div_e4m3x8(lo, s, rc, o2);
      o[0] = o2[0]; o[1] = o2[1];
      if (compiled) full_e4m3x8(hi, s, rc, o2);
      else div_e4m3x8(hi, s, rc, o2);
      o[2] = o2[0]; o[3] = o2[1];
    }
    if (q != nullptr && gr < R) {
      uint8_t *dst = q + gr * ldq + gc;
      if (vq && full) {
        *reinterpret_cast<uint4 *>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
      } else {
        for (int e = 0; e < 16; ++e)
          if (gc + e < C) dst[e] = (uint8_t)(o[e >> 2] >> (8 * (e & 3)));
      }
    }
    if (qT == nullptr) return;  // uniform over the CTA
#pragma unroll
    for (int i = 0; i < 4; ++i) *reinterpret_cast<uint32_t *>(&t[r][cq + 4 * i]) = o[i];
  }
  __syncthreads();
  {  // qT row c0 + tid/4 (a column of x), 16 values of rows r0 + (tid%4)*16 ..
    const int c = tid >> 2, rq = (tid & 3) * 16;
    const int64_t gr = c0 + c, gc = r0 + rq;
    if (gr >= C) return;
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int e = 0; e < 16; ++e) w[e >> 2] |= (uint32_t)t[rq + e][c] << (8 * (e & 3));
    uint8_t *dst = qT + gr * ldqT + gc;
    if (vqT && gc + 16 <= R) {
      *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      for (int e = 0; e < 16; ++e)
        if (gc + e < R) dst[e] = (uint8_t)(w[e >> 2] >> (8 * (e & 3)));
    }
  }
}

// dst[c][r] = src[r][c] for 1-byte elements (fp8 operands that cuBLASLt
// wants in the other major order).  A CTA moves a 64 x 64 byte tile through
// shared memory: 16-byte coalesced loads of source rows, 16-byte stores of
// destination rows.
__global__ void __launch_bounds__(kThreads)
transpose_b8_kernel(const uint8_t *src, int64_t rows, int64_t cols, int64_t lds, uint8_t *dst,
                    int64_t ldd, int vec) {
  __shared__ uint8_t t[64][64 + 4];
  const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
  const int tid = threadIdx.x;
  {  // load: row tid/4, 16 bytes at column (tid%4)*16
    const int r = tid >> 2, q = (tid & 3) * 16;
    const int64_t gr = r0 + r, gc = c0 + q;
    uint32_t w[4] = {0, 0, 0, 0};
    if (gr < rows) {
      if (vec && gc + 16 <= cols) {
        const uint4 v = ld_nc_v4(src + gr * lds + gc);
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
      } else {
        for (int e = 0; e < 16; ++e)
          if (gc + e < cols) w[e >> 2] |= (uint32_t)src[gr * lds + gc + e] << (8 * (e & 3));
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) *reinterpret_cast<uint32_t *>(&t[r][q + 4 * i]) = w[i];
  }
  __syncthreads();
  {  // store: destination row c = tid/4 (source column), 16 source rows
    const int c = tid >> 2, q = (tid & 3) * 16;
    const int64_t gr = c0 + c, gc = r0 + q;  // destination coordinates
    if (gr >= cols) return;
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int e = 0; e < 16; ++e) w[e >> 2] |= (uint32_t)t[q + e][c] << (8 * (e & 3));
    if (vec && gc + 16 <= rows) {
      *reinterpret_cast<uint4 *>(dst + gr * ldd + gc) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      for (int e = 0; e < 16; ++e)
        if (gc + e < rows) dst[gr * ldd + gc + e] = (w[e >> 2] >> (8 * (e & 3))) & 0xFFu;
    }
  }
}

}  // namespace bs

using namespace bs;

namespace {
int launch_err() { return cudaGetLastError() == cudaSuccess ? BS_OK : BS_ERR_LAUNCH; }
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

extern "C" int bs_fp8_scale(const void *x, int dtype, int64_t numel, uint32_t *amax_ws,
                            float *scale_out, void *stream) {
  const int compiled = (dtype & BS_FP8_COMPILED) != 0;
  dtype &= ~BS_FP8_COMPILED;
  if (dtype != BS_BF16 && dtype != BS_F32) return BS_ERR_DTYPE;
  if (numel < 0) return BS_ERR_SHAPE;
  if (!amax_ws || !scale_out || (numel > 0 && !x)) return BS_ERR_ARG;
  if (!aligned16(x)) return BS_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int eb = dtype == BS_BF16 ? 2 : 4;
  int64_t blocks = (numel * eb / 16 + kThreads - 1) / kThreads;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  const uint8_t *xb = static_cast<const uint8_t *>(x);
  if (dtype == BS_BF16) {
    amax_kernel<BS_BF16><<<(unsigned)blocks, kThreads, 0, st>>>(xb, numel, amax_ws);
    scale_kernel<BS_BF16><<<1, 1, 0, st>>>(amax_ws, scale_out, compiled);
  } else {
    amax_kernel<BS_F32><<<(unsigned)blocks, kThreads, 0, st>>>(xb, numel, amax_ws);
    scale_kernel<BS_F32><<<1, 1, 0, st>>>(amax_ws, scale_out, compiled);
  }
  return launch_err();
}

extern "C" int bs_fp8_scales_bias_relu(const void *z, int64_t M, int64_t N, int64_t ld,
                                       const void *bias, uint32_t *amax_ws, float *scale_h,
                                       float *scale_h2, int fp8_flags, void *stream) {
  if (M < 0 || N < 0 || ld < N) return BS_ERR_SHAPE;
  if (!amax_ws || !scale_h || !bias || (M > 0 && N > 0 && !z)) return BS_ERR_ARG;
  if (!aligned16(z) || !aligned16(bias)) return BS_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t blocks = (M * ((N + 7) / 8) + kThreads - 1) / kThreads;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  amax_bias_relu_kernel<<<(unsigned)blocks, kThreads, 0, st>>>(
      static_cast<const uint8_t *>(z), M, N, ld, static_cast<const uint8_t *>(bias), amax_ws);
  scales_relu2_kernel<<<1, 1, 0, st>>>(amax_ws, scale_h, scale_h2,
                                       (fp8_flags & BS_FP8_COMPILED) != 0);
  return launch_err();
}

extern "C" int bs_quantize_e4m3(const void *x, int dtype, int64_t numel, const float *scale,
                                uint8_t *q, void *stream) {
  const int compiled = (dtype & BS_FP8_COMPILED) != 0;
  dtype &= ~BS_FP8_COMPILED;
  if (dtype != BS_BF16 && dtype != BS_F32) return BS_ERR_DTYPE;
  if (numel < 0) return BS_ERR_SHAPE;
  if (numel == 0) return BS_OK;
  if (!x || !scale || !q) return BS_ERR_ARG;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7)) return BS_ERR_ALIGN;
  int64_t blocks = ((numel + 7) / 8 + kThreads - 1) / kThreads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t *xb = static_cast<const uint8_t *>(x);
  if (dtype == BS_BF16)
    quant_kernel<BS_BF16><<<(unsigned)blocks, kThreads, 0, st>>>(xb, numel, scale, q, compiled);
  else
    quant_kernel<BS_F32><<<(unsigned)blocks, kThreads, 0, st>>>(xb, numel, scale, q, compiled);
  return launch_err();
}

extern "C" int bs_transpose_b8(const void *src, int64_t rows, int64_t cols, int64_t ld_src,
                               void *dst, int64_t ld_dst, void *stream) {
  if (rows < 0 || cols < 0 || ld_src < cols || ld_dst < rows) return BS_ERR_SHAPE;
  if (rows == 0 || cols == 0) return BS_OK;
  if (!src || !dst) return BS_ERR_ARG;
  const int vec = aligned16(src) && aligned16(dst) && ld_src % 16 == 0 && ld_dst % 16 == 0;
  const dim3 grid((unsigned)((cols + 63) / 64), (unsigned)((rows + 63) / 64));
  if (grid.y > 65535) return BS_ERR_SHAPE;
  transpose_b8_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t *>(src), rows, cols, ld_src, static_cast<uint8_t *>(dst), ld_dst,
      vec);
  return launch_err();
}

extern "C" const char *bs_version(void) { return "bitsparse_b200 0.1 sm_100a"; }

extern "C" int bs_quantize_e4m3_2d(const void *x, int64_t R, int64_t C, int64_t ld,
                                   const float *scale, uint8_t *q, int64_t ldq, uint8_t *qT,
                                   int64_t ldqT, int fp8_flags, void *stream) {
  if (R < 0 || C < 0 || ld < C || (q && ldq < C) || (qT && ldqT < R)) return BS_ERR_SHAPE;
  if (R == 0 || C == 0 || (!q && !qT)) return BS_OK;
  if (!x || !scale) return BS_ERR_ARG;
  const dim3 grid((unsigned)((C + 63) / 64), (unsigned)((R + 63) / 64));
  if ((C + 63) / 64 > 0x7FFFFFFF || grid.y > 65535) return BS_ERR_SHAPE;
  const int vx = aligned16(x) && (ld * 2) % 16 == 0;
  const int vq = q && aligned16(q) && ldq % 16 == 0;
  const int vqT = qT && aligned16(qT) && ldqT % 16 == 0;
  quant2d_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t *>(x), R, C, ld, scale, q, ldq, qT, ldqT, vx, vq, vqT,
      (fp8_flags & BS_FP8_COMPILED) != 0);
  return launch_err();
}

__global__ void estimate_exact_kernel(const float *scale, int compiled, int *out) {
  const float s = *scale;
  const bool ok = e4m3_estimate_exact(s, quant_rcp(s), compiled != 0);
  if (threadIdx.x == 0) *out = ok ? 1 : 0;
}

extern "C" int bs_fp8_estimate_exact(const float *scale, int fp8_flags, int *out, void *stream) {
  if (!scale || !out) return BS_ERR_ARG;
  estimate_exact_kernel<<<1, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      scale, (fp8_flags & BS_FP8_COMPILED) != 0, out);
  return launch_err();
}
