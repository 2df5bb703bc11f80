// K2 -- reconstruct (unpack) and the backward mask kernels.
//
// Reference behaviour replaced (Maxzhu123/bitsparse):
//   _unpack_batch_kernel      lib_sparse/src/triton_kernels.py:158-241
//   unpack_relu2_batch_ scale lib_sparse/src/triton_operators.py:141-162
//   load_packed_at_indices    lib_sparse/src/bitpacking.py:37-55
//   _relu_grad_sparse_kernel  lib_sparse/src/triton_kernels.py:249-276
//   _relu2_grad_sparse_kernel lib_sparse/src/triton_kernels.py:288-330 (+ the
//                             host-side grad.mul_(scale), triton_operators.py:200-201)
//
// One CTA of 256 threads per tile.  The tile's value segment
// [prefix[t] + vals_offset, prefix[t+1] + vals_offset) is contiguous in the
// value stream, so it is fetched with aligned 16-byte loads into shared
// memory (raw) or as the 32-bit words covering its bit range (packed)
// while the bitmask is read and scanned; each thread then expands its
// 16-byte output chunk(s) from shared memory and writes them with one
// 16-byte store.  Every DRAM byte of the value stream, bitmask and output is
// touched once.  The reference's separate scale passes (output *= scale^2,
// grad *= scale) are fused with the reference's double rounding preserved.
#include "common.cuh"

namespace bs {

// Value segment staging capacity: 4096 values of up to 2 bytes, plus the
// alignment slack of the first 16-byte vector and one extra packed word.
constexpr int kStageBytes = kTileNumel * 2 + 64;

struct UnpackParams {
  const uint8_t *vals;
  const uint8_t *bitmask;
  const uint32_t *prefix;
  const int64_t *vals_offset;
  uint8_t *out;  // unpack: output; grad kernels: grad (in place)
  int64_t out_ld;
  int64_t first_m_tile, grid_n, K, batch_rows;
  const float *scale;
  float k;       // RELU2_SCALE
  int vals_v16;  // vals base 16-byte aligned
  int out_vec;   // out base + row stride allow 16-byte accesses
};

// Fetch tile `tile`'s value segment into smem.  Returns the index in
// `stage` (in elements for raw, in bits for packed) of the tile's first value.
template <int SDT, bool PACK>
__device__ __forceinline__ uint32_t stage_values(const UnpackParams &P, int64_t tile,
                                                 uint8_t *stage) {
  constexpr int SB = Elt<SDT>::bytes;
  const int64_t voff = P.vals_offset ? *P.vals_offset : 0;
  const uint32_t p0 = P.prefix[tile], p1 = P.prefix[tile + 1];
  uint32_t cnt = p1 - p0;
  if (cnt > (uint32_t)kTileNumel) cnt = kTileNumel;
  const int64_t base = (int64_t)p0 + voff;
  const int tid = threadIdx.x;
  if constexpr (!PACK) {
    constexpr int EPV = 16 / SB;
    const int64_t v0 = base / EPV;
    const int64_t nvec = cnt ? (base + cnt - 1) / EPV - v0 + 1 : 0;
    if (P.vals_v16) {
      for (int64_t i = tid; i < nvec; i += kThreads)
        *reinterpret_cast<uint4 *>(stage + 16 * i) = ld_nc_v4(P.vals + (v0 + i) * 16);
    } else {
      for (int64_t i = tid; i < nvec * 16; i += kThreads) {
        const int64_t byte = v0 * 16 + i;
        const int64_t e = byte / SB;
        stage[i] = (e >= base && e < base + cnt) ? P.vals[byte] : 0;
      }
    }
    return (uint32_t)(base - v0 * EPV);
  } else {
    constexpr int B = pack_bits<SDT>();
    const int64_t bit0 = base * B;
    const int64_t w0 = bit0 >> 5;
    const int64_t nw = cnt ? (((base + cnt) * B + 31) >> 5) - w0 : 0;
    const uint32_t *words = reinterpret_cast<const uint32_t *>(P.vals);
    uint32_t *sw = reinterpret_cast<uint32_t *>(stage);
    for (int64_t i = tid; i < nw; i += kThreads) sw[i] = __ldg(words + w0 + i);
    if (tid == 0) sw[nw] = 0;  // guard for two-word reads of the last value
    return (uint32_t)(bit0 - (w0 << 5));
  }
}

// Value `r` of the staged segment as raw stored bits.
template <int SDT, bool PACK>
__device__ __forceinline__ uint32_t staged_value(const uint8_t *stage, uint32_t first,
                                                 uint32_t r) {
  if constexpr (!PACK) {
    if constexpr (Elt<SDT>::bytes == 1) return stage[first + r];
    else return reinterpret_cast<const uint16_t *>(stage)[first + r];
  } else {
    constexpr int B = pack_bits<SDT>();
    const uint32_t bit = first + r * B;
    const uint32_t *sw = reinterpret_cast<const uint32_t *>(stage);
    const uint64_t two = (uint64_t)sw[bit >> 5] | ((uint64_t)sw[(bit >> 5) + 1] << 32);
    return (uint32_t)(two >> (bit & 31)) & ((1u << B) - 1u);
  }
}

// Block-wide exclusive scan of CH per-thread counts in (slot, warp, lane)
// order.  Returns each slot's exclusive offset in `ex`.
template <int CH>
__device__ __forceinline__ void block_excl_scan(const uint32_t (&cnt)[CH], uint32_t (&ex)[CH],
                                                uint32_t *s_wt) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t lex[CH];
#pragma unroll
  for (int s = 0; s < CH; ++s) {
    const uint32_t inc = warp_incl_scan(cnt[s]);
    lex[s] = inc - cnt[s];
    if (lane == 31) s_wt[s * 8 + warp] = inc;
  }
  __syncthreads();
  if (warp == 0) {
    constexpr int NW = CH * 8;
    const uint32_t v = lane < NW ? s_wt[lane] : 0;
    const uint32_t inc = warp_incl_scan(v);
    if (lane < NW) s_wt[lane] = inc - v;
  }
  __syncthreads();
#pragma unroll
  for (int s = 0; s < CH; ++s) ex[s] = s_wt[s * 8 + warp] + lex[s];
}

__device__ __forceinline__ int64_t tile_of_pid(const UnpackParams &P, int64_t pid) {
  return (P.first_m_tile + pid / P.grid_n) * P.grid_n + pid % P.grid_n;
}

// OUT: 0 = elements of SDT (plain reconstruct), 1 = bf16 k*r^2 (ReLU^2).
template <int SDT, bool PACK, int OUT, bool SCALE>
__global__ void __launch_bounds__(kThreads) unpack_kernel(const UnpackParams P) {
  constexpr int OB = OUT ? 2 : Elt<SDT>::bytes;  // output element bytes
  constexpr int VEC = 16 / OB;                   // output elements per chunk
  constexpr int CPR = kTileN / VEC, CPT = kTileNumel / VEC, CH = CPT / kThreads;
  __shared__ __align__(16) uint8_t stage[kStageBytes];
  __shared__ uint32_t s_wt[CH * 8];

  const int64_t pid = blockIdx.x;
  const int64_t tile = tile_of_pid(P, pid);
  const int tid = threadIdx.x;
  const uint32_t first = stage_values<SDT, PACK>(P, tile, stage);

  uint32_t m[CH], cnt[CH], ex[CH];
  const uint8_t *bm = P.bitmask + tile * kTileBytes;
#pragma unroll
  for (int s = 0; s < CH; ++s) {
    const int c = s * kThreads + tid;
    if constexpr (VEC == 8) m[s] = bm[c];
    else m[s] = reinterpret_cast<const uint16_t *>(bm)[c];
    cnt[s] = __popc(m[s]);
  }
  block_excl_scan<CH>(cnt, ex, s_wt);  // contains __syncthreads (stage ready)

  float s2 = 0.f;
  if constexpr (SCALE) {
    const float sc = *P.scale;
    s2 = bf16_bits_to_f32(f32_to_bf16_bits(sc * sc));
  }
  const int64_t row_t = (pid / P.grid_n) * kTileM, col_t = (pid % P.grid_n) * kTileN;
#pragma unroll
  for (int s = 0; s < CH; ++s) {
    const int c = s * kThreads + tid;
    const int row = c / CPR, cc = c % CPR;
    uint32_t w[4] = {0, 0, 0, 0};
    const uint32_t mm = m[s];
    uint32_t r = ex[s];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {  // static indices keep w[] in registers
      if (!((mm >> e) & 1u)) continue;
      uint32_t v = staged_value<SDT, PACK>(stage, first, r++);
      if constexpr (OUT == 1) {
        if constexpr (SDT == BS_BF16) {
          const float x = bf16_bits_to_f32(v);
          const float kx = bf16_bits_to_f32(f32_to_bf16_bits(P.k * x));
          v = f32_to_bf16_bits(kx * x);
        } else {
          const float x = store_bits_to_f32<SDT>(v);
          v = f32_to_bf16_bits(P.k * x * x);
        }
        if constexpr (SCALE) v = f32_to_bf16_bits(bf16_bits_to_f32(v) * s2);
      }
      if constexpr (OB == 1) w[e >> 2] |= v << (8 * (e & 3));
      else w[e >> 1] |= v << (16 * (e & 1));
    }
    const int64_t grow = row_t + row, gcol = col_t + cc * VEC;
    if (grow >= P.batch_rows) continue;
    uint8_t *dst = P.out + (grow * P.out_ld + gcol) * OB;
    if (P.out_vec && gcol + VEC <= P.K) {
      st_v4(dst, make_uint4(w[0], w[1], w[2], w[3]));
    } else {
      for (int e = 0; e < VEC; ++e) {
        if (gcol + e >= P.K) break;
        if constexpr (OB == 1) dst[e] = (w[e >> 2] >> (8 * (e & 3))) & 0xFFu;
        else reinterpret_cast<uint16_t *>(dst)[e] = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
      }
    }
  }
}

// grad <- bit ? grad : 0.  GB = grad element bytes (2 bf16, 4 fp32); one chunk
// = 8 elements = one bitmask byte.
template <int GB>
__global__ void __launch_bounds__(kThreads) mask_kernel(const UnpackParams P) {
  constexpr int CH = 2;  // 512 chunks of 8 per tile
  const int64_t tile = blockIdx.x;
  const int64_t row_t = (tile / P.grid_n) * kTileM, col_t = (tile % P.grid_n) * kTileN;
  const uint8_t *bm = P.bitmask + tile * kTileBytes;
#pragma unroll
  for (int s = 0; s < CH; ++s) {
    const int c = s * kThreads + threadIdx.x;
    const int row = c / 8, cc = c % 8;
    const int64_t grow = row_t + row, gcol = col_t + cc * 8;
    if (grow >= P.batch_rows) continue;
    const uint32_t mb = bm[c];
    uint8_t *g = P.out + (grow * P.out_ld + gcol) * GB;
    if (P.out_vec && gcol + 8 <= P.K) {
      if (mb == 0xFFu) continue;  // nothing to clear
#pragma unroll
      for (int l = 0; l < GB / 2; ++l) {
        uint4 v = *reinterpret_cast<const uint4 *>(g + 16 * l);
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if constexpr (GB == 2) {
            const int e0 = l * 8 + 2 * i;
            const uint32_t keep = ((mb >> e0) & 1u ? 0xFFFFu : 0u) |
                                  ((mb >> (e0 + 1)) & 1u ? 0xFFFF0000u : 0u);
            w[i] &= keep;
          } else {
            const int e = l * 4 + i;
            if (!((mb >> e) & 1u)) w[i] = 0;
          }
        }
        st_v4(g + 16 * l, make_uint4(w[0], w[1], w[2], w[3]));
      }
    } else {
      for (int e = 0; e < 8; ++e) {
        if (gcol + e >= P.K) break;
        if (!((mb >> e) & 1u)) {
          if constexpr (GB == 2) reinterpret_cast<uint16_t *>(g)[e] = 0;
          else reinterpret_cast<uint32_t *>(g)[e] = 0;
        }
      }
    }
  }
}

// grad <- bit ? bf16(grad * (2 k r)) : 0, then (SCALE) bf16(grad * bf16(scale)).
template <int SDT, bool PACK, bool SCALE>
__global__ void __launch_bounds__(kThreads) relu2_grad_kernel(const UnpackParams P) {
  constexpr int CH = 2, CPR = 8;
  __shared__ __align__(16) uint8_t stage[kStageBytes];
  __shared__ uint32_t s_wt[CH * 8];
  const int64_t tile = blockIdx.x;
  const int tid = threadIdx.x;
  const uint32_t first = stage_values<SDT, PACK>(P, tile, stage);
  const uint8_t *bm = P.bitmask + tile * kTileBytes;
  uint32_t m[CH], cnt[CH], ex[CH];
#pragma unroll
  for (int s = 0; s < CH; ++s) {
    m[s] = bm[s * kThreads + tid];
    cnt[s] = __popc(m[s]);
  }
  block_excl_scan<CH>(cnt, ex, s_wt);
  float sb = 0.f;
  if constexpr (SCALE) sb = bf16_bits_to_f32(f32_to_bf16_bits(*P.scale));
  const float two_k = 2.0f * P.k;
  const int64_t row_t = (tile / P.grid_n) * kTileM, col_t = (tile % P.grid_n) * kTileN;
#pragma unroll
  for (int s = 0; s < CH; ++s) {
    const int c = s * kThreads + tid;
    const int row = c / CPR, cc = c % CPR;
    const int64_t grow = row_t + row, gcol = col_t + cc * 8;
    if (grow >= P.batch_rows) continue;
    uint16_t *g = reinterpret_cast<uint16_t *>(P.out + (grow * P.out_ld + gcol) * 2);
    uint32_t gv[8];
    const bool vec = P.out_vec && gcol + 8 <= P.K;
    if (vec) {
      const uint4 v = *reinterpret_cast<const uint4 *>(g);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) gv[e] = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) gv[e] = (gcol + e < P.K) ? g[e] : 0u;
    }
    uint32_t r = ex[s];
    uint32_t o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if ((m[s] >> e) & 1u) {
        const float rv = store_bits_to_f32<SDT>(staged_value<SDT, PACK>(stage, first, r++));
        uint32_t y = f32_to_bf16_bits(bf16_bits_to_f32(gv[e]) * (two_k * rv));
        if constexpr (SCALE) y = f32_to_bf16_bits(bf16_bits_to_f32(y) * sb);
        o[e] = y;
      } else {
        o[e] = 0;
      }
    }
    if (vec) {
      st_v4(g, make_uint4(o[0] | (o[1] << 16), o[2] | (o[3] << 16), o[4] | (o[5] << 16),
                          o[6] | (o[7] << 16)));
    } else {
      for (int e = 0; e < 8; ++e)
        if (gcol + e < P.K) g[e] = (uint16_t)o[e];
    }
  }
}

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
__global__ void scale_kernel(uint32_t *amax_ws, float *scale_out) {
  const float amax = __uint_as_float(*amax_ws);
  float s = __fdiv_rn(amax, 448.0f);
  if constexpr (DT == BS_BF16) s = bf16_bits_to_f32(f32_to_bf16_bits(s));
  *scale_out = fmaxf(s, 1e-9f);  // clamp(min=1e-9)
  *amax_ws = 0u;
}

// q = e4m3(x / scale) over a flat tensor (the quantise half of to_fp8).
template <int DT>
__global__ void __launch_bounds__(kThreads)
quant_kernel(const uint8_t *x, int64_t n, const float *scale, uint8_t *q) {
  const float s = *scale;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
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
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float xv = DT == BS_BF16 ? bf16_bits_to_f32(b[e]) : __uint_as_float(b[e]);
      float y = __fdiv_rn(xv, s);
      if constexpr (DT == BS_BF16) y = bf16_bits_to_f32(f32_to_bf16_bits(y));
      o[e >> 2] |= f32_to_e4m3_bits(y) << (8 * (e & 3));
    }
    if (full) {
      *reinterpret_cast<uint2 *>(q + e0) = make_uint2(o[0], o[1]);
    } else {
      for (int e = 0; e < 8 && e0 + e < n; ++e) q[e0 + e] = (o[e >> 2] >> (8 * (e & 3))) & 0xFFu;
    }
  }
}

}  // namespace bs

using namespace bs;

namespace {

int launch_err() { return cudaGetLastError() == cudaSuccess ? BS_OK : BS_ERR_LAUNCH; }

template <int SDT, bool PACK>
int unpack_disp2(const UnpackParams &P, int64_t ntiles, int relu2, bool scale, cudaStream_t st) {
  const dim3 g((unsigned)ntiles);
  if (!relu2) unpack_kernel<SDT, PACK, 0, false><<<g, kThreads, 0, st>>>(P);
  else if (scale) unpack_kernel<SDT, PACK, 1, true><<<g, kThreads, 0, st>>>(P);
  else unpack_kernel<SDT, PACK, 1, false><<<g, kThreads, 0, st>>>(P);
  return launch_err();
}

template <int SDT>
int unpack_disp(const UnpackParams &P, int pack, int64_t ntiles, int relu2, bool scale,
                cudaStream_t st) {
  return pack ? unpack_disp2<SDT, true>(P, ntiles, relu2, scale, st)
              : unpack_disp2<SDT, false>(P, ntiles, relu2, scale, st);
}

template <int SDT, bool PACK>
int relu2g_disp2(const UnpackParams &P, int64_t ntiles, bool scale, cudaStream_t st) {
  const dim3 g((unsigned)ntiles);
  if (scale) relu2_grad_kernel<SDT, PACK, true><<<g, kThreads, 0, st>>>(P);
  else relu2_grad_kernel<SDT, PACK, false><<<g, kThreads, 0, st>>>(P);
  return launch_err();
}

template <int SDT>
int relu2g_disp(const UnpackParams &P, int pack, int64_t ntiles, bool scale, cudaStream_t st) {
  return pack ? relu2g_disp2<SDT, true>(P, ntiles, scale, st)
              : relu2g_disp2<SDT, false>(P, ntiles, scale, st);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" int bs_unpack(const void *vals, const uint8_t *bitmask, const uint32_t *prefix,
                         const int64_t *vals_offset, int store_dtype, int pack_sbit, void *out,
                         int64_t out_ld, int64_t first_m_tile, int64_t grid_n, int64_t K,
                         int64_t batch_rows, int64_t num_tiles_in_batch, int relu2,
                         const float *scale, void *stream) {
  if (store_dtype != BS_BF16 && store_dtype != BS_E4M3 && store_dtype != BS_E5M2)
    return BS_ERR_DTYPE;
  if (num_tiles_in_batch < 0 || first_m_tile < 0 || grid_n < 0 || K < 0 || batch_rows < 0 ||
      out_ld < K)
    return BS_ERR_SHAPE;
  if (num_tiles_in_batch == 0) return BS_OK;
  if (grid_n == 0 || num_tiles_in_batch > ((int64_t)1 << 31)) return BS_ERR_SHAPE;
  if (!bitmask || !prefix || !out) return BS_ERR_ARG;
  if (pack_sbit && (reinterpret_cast<uintptr_t>(vals) & 3)) return BS_ERR_ALIGN;
  if (!relu2 && scale) return BS_ERR_ARG;
  UnpackParams P{};
  P.vals = static_cast<const uint8_t *>(vals);
  P.bitmask = bitmask;
  P.prefix = prefix;
  P.vals_offset = vals_offset;
  P.out = static_cast<uint8_t *>(out);
  P.out_ld = out_ld;
  P.first_m_tile = first_m_tile;
  P.grid_n = grid_n;
  P.K = K;
  P.batch_rows = batch_rows;
  P.scale = scale;
  P.k = 1.0f;
  const int ob = relu2 ? 2 : (store_dtype == BS_BF16 ? 2 : 1);
  P.vals_v16 = aligned16(vals);
  P.out_vec = aligned16(out) && ((out_ld * ob) % 16 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (store_dtype) {
    case BS_BF16: return unpack_disp<BS_BF16>(P, pack_sbit, num_tiles_in_batch, relu2, scale, st);
    case BS_E4M3: return unpack_disp<BS_E4M3>(P, pack_sbit, num_tiles_in_batch, relu2, scale, st);
    default: return unpack_disp<BS_E5M2>(P, pack_sbit, num_tiles_in_batch, relu2, scale, st);
  }
}

extern "C" int bs_mask_with_bitmask(void *grad, int grad_dtype, int64_t M, int64_t N,
                                    int64_t ld, const uint8_t *bitmask, void *stream) {
  if (grad_dtype != BS_BF16 && grad_dtype != BS_F32) return BS_ERR_DTYPE;
  if (M < 0 || N < 0 || ld < N) return BS_ERR_SHAPE;
  const int64_t gm = (M + 63) / 64, gn = (N + 63) / 64;
  if (gm * gn == 0) return BS_OK;
  if (!grad || !bitmask) return BS_ERR_ARG;
  UnpackParams P{};
  P.bitmask = bitmask;
  P.out = static_cast<uint8_t *>(grad);
  P.out_ld = ld;
  P.grid_n = gn;
  P.K = N;
  P.batch_rows = M;
  const int gb = grad_dtype == BS_BF16 ? 2 : 4;
  P.out_vec = aligned16(grad) && ((ld * gb) % 16 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (gb == 2) mask_kernel<2><<<(unsigned)(gm * gn), kThreads, 0, st>>>(P);
  else mask_kernel<4><<<(unsigned)(gm * gn), kThreads, 0, st>>>(P);
  return launch_err();
}

extern "C" int bs_relu2_grad(void *grad, int grad_dtype, int64_t M, int64_t N, int64_t ld,
                             const void *vals, const uint8_t *bitmask, const uint32_t *prefix,
                             const int64_t *vals_offset, int store_dtype, int pack_sbit,
                             const float *scale, void *stream) {
  if (grad_dtype != BS_BF16) return BS_ERR_DTYPE;
  if (store_dtype != BS_BF16 && store_dtype != BS_E4M3 && store_dtype != BS_E5M2)
    return BS_ERR_DTYPE;
  if (M < 0 || N < 0 || ld < N) return BS_ERR_SHAPE;
  const int64_t gm = (M + 63) / 64, gn = (N + 63) / 64;
  if (gm * gn == 0) return BS_OK;
  if (!grad || !bitmask || !prefix) return BS_ERR_ARG;
  if (pack_sbit && (reinterpret_cast<uintptr_t>(vals) & 3)) return BS_ERR_ALIGN;
  UnpackParams P{};
  P.vals = static_cast<const uint8_t *>(vals);
  P.bitmask = bitmask;
  P.prefix = prefix;
  P.vals_offset = vals_offset;
  P.out = static_cast<uint8_t *>(grad);
  P.out_ld = ld;
  P.first_m_tile = 0;
  P.grid_n = gn;
  P.K = N;
  P.batch_rows = M;
  P.scale = scale;
  P.k = 1.0f;
  P.vals_v16 = aligned16(vals);
  P.out_vec = aligned16(grad) && ((ld * 2) % 16 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool sc = scale != nullptr;
  switch (store_dtype) {
    case BS_BF16: return relu2g_disp<BS_BF16>(P, pack_sbit, gm * gn, sc, st);
    case BS_E4M3: return relu2g_disp<BS_E4M3>(P, pack_sbit, gm * gn, sc, st);
    default: return relu2g_disp<BS_E5M2>(P, pack_sbit, gm * gn, sc, st);
  }
}

extern "C" int bs_fp8_scale(const void *x, int dtype, int64_t numel, uint32_t *amax_ws,
                            float *scale_out, void *stream) {
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
    scale_kernel<BS_BF16><<<1, 1, 0, st>>>(amax_ws, scale_out);
  } else {
    amax_kernel<BS_F32><<<(unsigned)blocks, kThreads, 0, st>>>(xb, numel, amax_ws);
    scale_kernel<BS_F32><<<1, 1, 0, st>>>(amax_ws, scale_out);
  }
  return launch_err();
}

extern "C" int bs_quantize_e4m3(const void *x, int dtype, int64_t numel, const float *scale,
                                uint8_t *q, void *stream) {
  if (dtype != BS_BF16 && dtype != BS_F32) return BS_ERR_DTYPE;
  if (numel < 0) return BS_ERR_SHAPE;
  if (numel == 0) return BS_OK;
  if (!x || !scale || !q) return BS_ERR_ARG;
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7)) return BS_ERR_ALIGN;
  int64_t blocks = ((numel + 7) / 8 + kThreads - 1) / kThreads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t *xb = static_cast<const uint8_t *>(x);
  if (dtype == BS_BF16) quant_kernel<BS_BF16><<<(unsigned)blocks, kThreads, 0, st>>>(xb, numel, scale, q);
  else quant_kernel<BS_F32><<<(unsigned)blocks, kThreads, 0, st>>>(xb, numel, scale, q);
  return launch_err();
}

extern "C" const char *bs_version(void) { return "bitsparse_b200 0.1 sm_100a"; }
