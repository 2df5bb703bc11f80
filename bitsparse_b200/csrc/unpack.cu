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
// A CTA of 256 threads handles UT = 2 consecutive tiles of the batch.  Their
// value segment [prefix[t0] + vals_offset, prefix[t0 + 2] + vals_offset) is
// contiguous in the stream, so it is fetched into shared memory with aligned
// 16-byte loads (raw) or as the 32-bit words covering its bit range (packed)
// while the bitmask is read and scanned.  Each thread then expands 32-byte
// output chunks (16 bf16 / 32 fp8 elements of one tile row) from shared
// memory and writes each with one 256-bit store.  Every DRAM byte of the
// stream, bitmask and output is touched once.  The reference's separate
// scale passes (output *= scale^2, grad *= scale) are fused, keeping the
// reference's double rounding.
#include <cstdlib>
#include <type_traits>

#include "common.cuh"

namespace bs {

constexpr int kUT = 2;  // tiles per CTA
// Value segment staging: 2 tiles x 4096 values x up to 2 bytes, plus the
// first vector's alignment slack and a guard word for packed decoding.
constexpr int kStageBytes = kUT * kTileNumel * 2 + 64;

struct UnpackParams {
  const uint8_t *vals;
  const uint8_t *bitmask;
  const uint32_t *prefix;
  const int64_t *vals_offset;
  uint8_t *out;  // unpack: output; grad kernels: grad (in place)
  int64_t out_ld;
  int64_t first_tile;  // tile id of batch position 0 (first_m_tile * grid_n)
  int64_t ntiles;      // tiles in the batch
  int64_t grid_n, K, batch_rows;
  const float *scale;
  float k;       // RELU2_SCALE
  const float *qscale;  // OUT 2: to_fp8 scale of the ReLU^2 reconstruction
  int qcompiled;  // OUT 2: to_fp8 as the reference's compiled version (BS_FP8_COMPILED)
  int vals_v16;  // vals base 16-byte aligned
  int out_v32;   // out base + row stride allow 32-byte accesses
  // plain reconstruct: a warp scatters only the set values of its chunks
  // when none holds more than this many (else every element reads its rank)
  uint32_t scatter_max;
  // OUT 3: the per-tile scales of an e4m3 tensor compressed in per-tile
  // scale mode (one per tile of the whole tensor)
  const float *tile_scales;
};

__device__ __forceinline__ void st_v8(void *p, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(w[0]),
               "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}
__device__ __forceinline__ void ld_v8(const void *p, uint32_t (&w)[8]) {
  asm volatile("ld.global.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]),
                 "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}

// Fetch the value segment of tiles [t0, t0 + nt) into smem.  Returns the
// position in `stage` (elements for raw, bits for packed) of the first value.
template <int SDT, bool PACK>
__device__ __forceinline__ uint32_t stage_values(const UnpackParams &P, int64_t t0, int nt,
                                                 uint8_t *stage) {
  constexpr int SB = Elt<SDT>::bytes;
  const int64_t voff = P.vals_offset ? *P.vals_offset : 0;
  const uint32_t p0 = P.prefix[t0], p1 = P.prefix[t0 + nt];
  uint32_t cnt = p1 - p0;
  if (cnt > (uint32_t)(kUT * kTileNumel)) cnt = kUT * kTileNumel;
  const int64_t base = (int64_t)p0 + voff;
  const int tid = threadIdx.x;
  if constexpr (!PACK) {
    constexpr int EPV = 16 / SB;
    const int64_t v0 = base / EPV;
    const int64_t nvec = cnt ? (base + cnt - 1) / EPV - v0 + 1 : 0;
    if (P.vals_v16) {
      // all of this thread's vectors are loaded before any is stored
      constexpr int kPer = (kStageBytes / 16 + kThreads - 1) / kThreads;
      uint4 v[kPer];
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int64_t i = tid + (int64_t)k * kThreads;
        if (i < nvec) v[k] = ld_nc_v4(P.vals + (v0 + i) * 16);
      }
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int64_t i = tid + (int64_t)k * kThreads;
        if (i < nvec) *reinterpret_cast<uint4 *>(stage + 16 * i) = v[k];
      }
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
    constexpr int kPer = (kStageBytes / 4 + kThreads - 1) / kThreads;
    uint32_t v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int64_t i = tid + (int64_t)k * kThreads;
      if (i < nw) v[k] = __ldg(words + w0 + i);
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int64_t i = tid + (int64_t)k * kThreads;
      if (i < nw) sw[i] = v[k];
    }
    if (tid == 0) sw[nw] = 0;  // guard for the two-word read of the last value
    return (uint32_t)(bit0 - (w0 << 5));
  }
}

// Value r of the staged segment, as raw stored bits.
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

// Block-wide exclusive scan of S per-thread counts in (slot, warp, lane) order.
// One barrier: after it every warp reads all S * 8 warp totals and adds up
// those before its own (slot, warp) with one warp reduction per slot (no
// second-level scan by one warp, no second barrier).  The caller passes a
// barrier before s_wt is written again.
template <int S>
__device__ __forceinline__ void block_excl_scan(const uint32_t (&cnt)[S], uint32_t (&ex)[S],
                                                uint32_t *s_wt) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NW = S * 8;
  static_assert(NW <= 32, "a warp holds the warp totals");
  uint32_t lex[S];
  if constexpr (S == 2) {
    // both slots in one scan: 16-bit fields (a warp's slot total is at most
    // 32 chunks x 32 values, so the low field never carries)
    const uint32_t packed = cnt[0] | (cnt[1] << 16);
    const uint32_t inc = warp_incl_scan(packed);
    lex[0] = (inc & 0xFFFFu) - cnt[0];
    lex[1] = (inc >> 16) - cnt[1];
    if (lane == 31) {
      s_wt[warp] = inc & 0xFFFFu;
      s_wt[8 + warp] = inc >> 16;
    }
  } else {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const uint32_t inc = warp_incl_scan(cnt[s]);
      lex[s] = inc - cnt[s];
      if (lane == 31) s_wt[s * 8 + warp] = inc;
    }
  }
  __syncthreads();
  const uint32_t t = lane < NW ? s_wt[lane] : 0u;
#pragma unroll
  for (int s = 0; s < S; ++s)
    ex[s] = __reduce_add_sync(0xFFFFFFFFu, lane < s * 8 + warp ? t : 0u) + lex[s];
}

// Chunk geometry for 32-byte chunks of OB-byte elements.
template <int OB>
struct Chunk {
  static constexpr int VEC = 32 / OB;             // elements per chunk
  static constexpr int CPR = kTileN / VEC;        // chunks per tile row
  static constexpr int CPT = kTileNumel / VEC;    // chunks per tile
  static constexpr int S = kUT * CPT / kThreads;  // slots per thread
};

template <int VEC>
__device__ __forceinline__ uint32_t load_mask(const uint8_t *bm) {
  if constexpr (VEC == 8) return *bm;
  else if constexpr (VEC == 16) return *reinterpret_cast<const uint16_t *>(bm);
  else return *reinterpret_cast<const uint32_t *>(bm);
}

__device__ __forceinline__ int tiles_here(const UnpackParams &P, int64_t pid0) {
  const int64_t left = P.ntiles - pid0;
  return (int)(left < kUT ? left : kUT);
}

// Grid position of the CTA's tiles: one division for its first tile, then a
// wrapping step per tile (a 64-bit divide per chunk costs ~70 instructions).
struct PidPos {
  int64_t r0, c0, gn;
  // batches hold < 2^31 tiles (checked on the host): a 32-bit division
  __device__ __forceinline__ PidPos(int64_t pid0, int64_t grid_n) : gn(grid_n) {
    const uint32_t p = (uint32_t)pid0, n = (uint32_t)grid_n;
    const uint32_t q = p / n;
    r0 = q;
    c0 = p - q * n;
  }
  __device__ __forceinline__ void pos(int j, int64_t &tr, int64_t &tc) const {
    tr = r0;
    tc = c0 + j;
#pragma unroll
    for (int i = 0; i < kUT - 1; ++i)
      if (tc >= gn) { tc -= gn; ++tr; }
  }
};

// The ReLU^2 output for one stored code v (OUT 1: bf16 bits; OUT 2: e4m3
// bits), with the roundings of the reference's kernel and of to_fp8.
template <int SDT, int OUT, bool SCALE>
__device__ __forceinline__ uint32_t relu2_out(const UnpackParams &P, uint32_t v) {
  if constexpr (SDT == BS_BF16) {
    // bf16 * bf16 in bf16 (triton_kernels.py:238): k*v rounded, then *v
    const float x = bf16_bits_to_f32(v);
    const float kx = bf16_bits_to_f32(f32_to_bf16_bits(P.k * x));
    v = f32_to_bf16_bits(kx * x);
  } else {
    const float x = store_bits_to_f32<SDT>(v);  // fp8 squares in fp32 (:234-236)
    v = f32_to_bf16_bits(P.k * x * x);
  }
  if constexpr (SCALE) {
    const float sc = *P.scale;
    const float s2 = bf16_bits_to_f32(f32_to_bf16_bits(sc * sc));  // scale.square() in bf16
    v = f32_to_bf16_bits(bf16_bits_to_f32(v) * s2);
  }
  if constexpr (OUT == 2) {  // to_fp8's quantiser on the bf16 tensor (eager or compiled)
    const float qs = *P.qscale;
    v = P.qcompiled ? e4m3_compiled(bf16_bits_to_f32(v), qs, quant_rcp(qs))
                    : div_e4m3x2(bf16_bits_to_f32(v), 0.f, qs, quant_rcp(qs)) & 0xFFu;
  }
  return v;
}

// OUT: 0 = elements of SDT (plain reconstruct), 1 = bf16 k*r^2 (ReLU^2),
// 2 = the ReLU^2 reconstruction quantised to e4m3 with *qscale (to_fp8's
// quantiser) and written transposed (out is [K, batch_rows]) -- the B
// operand of the fp8 dW GEMM in the column-major order cuBLASLt wants;
// 3 = bf16(value(code) * scale of its tile), the dequantised tensor of the
// per-tile scale mode.
template <int SDT, bool PACK, int OUT, bool SCALE>
__global__ void __launch_bounds__(kThreads) unpack_kernel(const UnpackParams P) {
  constexpr int OB = (OUT == 1 || OUT == 3) ? 2 : (OUT == 2 ? 1 : Elt<SDT>::bytes);  // output bytes
  using G = Chunk<OB>;
  constexpr int kTP = 80;  // OUT 2: pitch of a transposed tile column in smem
  __shared__ __align__(16) uint8_t stage[kStageBytes];
  __shared__ uint32_t s_wt[G::S * 8];
  __shared__ __align__(16) uint8_t tstage[OUT == 2 ? kUT * kTileN * kTP : 16];
  // fp8 storage: the ReLU^2 output is a function of the 8-bit code alone, so
  // each CTA tabulates it once (256 codes, one per thread) and the element
  // loop becomes a table lookup.
  constexpr bool LUT = SDT != BS_BF16 && OUT >= 1;
  // OUT 2 tabulates 8-bit codes: a byte table spreads its 256 entries over
  // 64 words, so random lookups of a warp collide in fewer banks
  using LutT = typename std::conditional<OUT == 2, uint8_t, uint32_t>::type;
  __shared__ LutT lut[LUT ? 256 : 1];
  static_assert(!LUT || kThreads == 256, "one table entry per thread");

  const int64_t pid0 = (int64_t)blockIdx.x * kUT;
  const int nt = tiles_here(P, pid0);
  const PidPos pp(pid0, P.grid_n);
  const int tid = threadIdx.x;
  if constexpr (LUT) {
    if constexpr (OUT == 3) lut[tid] = __float_as_uint(store_bits_to_f32<SDT>((uint32_t)tid));
    else lut[tid] = (LutT)relu2_out<SDT, OUT, SCALE>(P, tid);
  }
  uint32_t m[G::S], cnt[G::S], ex[G::S];
#pragma unroll
  for (int s = 0; s < G::S; ++s) {  // masks first: independent of the values
    const int c = s * kThreads + tid;
    const int j = c / G::CPT, cc = c % G::CPT;
    m[s] = 0;
    if (j < nt)
      m[s] = load_mask<G::VEC>(P.bitmask + (P.first_tile + pid0 + j) * kTileBytes +
                               cc * (G::VEC / 8));
  }
  const uint32_t first = stage_values<SDT, PACK>(P, P.first_tile + pid0, nt, stage);
#pragma unroll
  for (int s = 0; s < G::S; ++s) cnt[s] = __popc(m[s]);
  block_excl_scan<G::S>(cnt, ex, s_wt);  // its barriers also publish the stage and table
#pragma unroll
  for (int s = 0; s < G::S; ++s) {
    const int c = s * kThreads + tid;
    const int j = c / G::CPT, cc = c % G::CPT;
    if (j >= nt) continue;
    const int row = cc / G::CPR, colc = cc % G::CPR;
    int64_t tr, tc;
    pp.pos(j, tr, tc);
    const int64_t grow = tr * kTileM + row;
    const int64_t gcol = tc * kTileN + colc * G::VEC;
    if (grow >= P.batch_rows) continue;
    uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const uint32_t mm = m[s];
    uint32_t r = ex[s];
    // OUT 3: this chunk's tile scale
    const float tsc = OUT == 3 ? P.tile_scales[P.first_tile + pid0 + j] : 1.f;
    if constexpr ((OUT == 0 || LUT) && !PACK) {
      // Branch-free expand: every element loads the value at its rank (the
      // stage has slack past the last value) and keeps it only if its bit
      // is set; divergent per-element branches cost more than the loads.
#pragma unroll
      for (int e = 0; e < G::VEC; ++e) {
        const uint32_t bit = (mm >> e) & 1u;
        uint32_t v = staged_value<SDT, PACK>(stage, first, r);
        if constexpr (LUT) v = lut[v];
        if constexpr (OUT == 3) v = f32_to_bf16_bits(__uint_as_float(v) * tsc);
        v &= 0u - bit;
        r += bit;
        if constexpr (OB == 1) w[e >> 2] |= v << (8 * (e & 3));
        else w[e >> 1] |= v << (16 * (e & 1));
      }
    }
#pragma unroll
    for (int e = 0; e < G::VEC; ++e) {  // static indices keep w[] in registers
      if constexpr ((OUT == 0 || LUT) && !PACK) break;
      if (!((mm >> e) & 1u)) continue;
      uint32_t v = staged_value<SDT, PACK>(stage, first, r++);
      if constexpr (LUT) v = lut[v];
      else if constexpr (OUT >= 1) v = relu2_out<SDT, OUT, SCALE>(P, v);
      if constexpr (OUT == 3) v = f32_to_bf16_bits(__uint_as_float(v) * tsc);
      if constexpr (OB == 1) w[e >> 2] |= v << (8 * (e & 3));
      else w[e >> 1] |= v << (16 * (e & 1));
    }
    if constexpr (OUT == 2) {  // into the transposed staging tile: column (colc*32+e), row
#pragma unroll
      for (int e = 0; e < G::VEC; ++e)
        tstage[(j * kTileN + colc * G::VEC + e) * kTP + row] = (uint8_t)(w[e >> 2] >> (8 * (e & 3)));
      continue;
    }
    uint8_t *dst = P.out + (grow * P.out_ld + gcol) * OB;
    if (P.out_v32 && gcol + G::VEC <= P.K) {
      st_v8(dst, w);
    } else {
      for (int e = 0; e < G::VEC; ++e) {
        if (gcol + e >= P.K) break;
        if constexpr (OB == 1) dst[e] = (w[e >> 2] >> (8 * (e & 3))) & 0xFFu;
        else reinterpret_cast<uint16_t *>(dst)[e] = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
      }
    }
  }
  if constexpr (OUT == 2) {
    // each tile leaves as 64 rows (its columns) of 64 bytes (its rows):
    // thread -> column tid / 4, rows 16 * (tid % 4) .. + 15, one 16-byte store
    __syncthreads();
    const int c = tid >> 2, r0 = (tid & 3) * 16;
    for (int j = 0; j < nt; ++j) {
      int64_t tr, tc;
      pp.pos(j, tr, tc);
      const int64_t ocol = tc * kTileN + c;    // output row  (a column of the tensor)
      const int64_t orow = tr * kTileM + r0;   // output column (a row of the tensor)
      if (ocol >= P.K || orow >= P.batch_rows) continue;
      const uint4 v = *reinterpret_cast<const uint4 *>(tstage + (j * kTileN + c) * kTP + r0);
      uint8_t *dst = P.out + ocol * P.out_ld + orow;
      if (P.out_v32 && orow + 16 <= P.batch_rows) {
        *reinterpret_cast<uint4 *>(dst) = v;
      } else {
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
        for (int e = 0; e < 16 && orow + e < P.batch_rows; ++e)
          dst[e] = (uint8_t)(w4[e >> 2] >> (8 * (e & 3)));
      }
    }
  }
}

// grad <- bit ? grad : 0 over 32-byte chunks (16 bf16 or 8 fp32 elements).
template <int GB>
__global__ void __launch_bounds__(kThreads) mask_kernel(const UnpackParams P) {
  using G = Chunk<GB>;
  const int64_t pid0 = (int64_t)blockIdx.x * kUT;
  const int nt = tiles_here(P, pid0);
  const PidPos pp(pid0, P.grid_n);
#pragma unroll
  for (int s = 0; s < G::S; ++s) {
    const int c = s * kThreads + threadIdx.x;
    const int j = c / G::CPT, cc = c % G::CPT;
    if (j >= nt) continue;
    const int64_t tile = pid0 + j;
    const int row = cc / G::CPR, colc = cc % G::CPR;
    int64_t tr, tc;
    pp.pos(j, tr, tc);
    const int64_t grow = tr * kTileM + row;
    const int64_t gcol = tc * kTileN + colc * G::VEC;
    if (grow >= P.batch_rows) continue;
    const uint32_t mb = load_mask<G::VEC>(P.bitmask + tile * kTileBytes + cc * (G::VEC / 8));
    constexpr uint32_t full = G::VEC == 16 ? 0xFFFFu : 0xFFu;
    uint8_t *g = P.out + (grow * P.out_ld + gcol) * GB;
    if (P.out_v32 && gcol + G::VEC <= P.K) {
      if (mb == full) continue;  // nothing to clear
      uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (mb) ld_v8(g, w);       // all-zero mask: the gradient need not be read
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if constexpr (GB == 2) {
          const uint32_t two = (mb >> (2 * i)) & 3u;
          w[i] &= (two & 1u ? 0xFFFFu : 0u) | (two & 2u ? 0xFFFF0000u : 0u);
        } else {
          if (!((mb >> i) & 1u)) w[i] = 0;
        }
      }
      st_v8(g, w);
    } else {
      for (int e = 0; e < G::VEC; ++e) {
        if (gcol + e >= P.K) break;
        if (!((mb >> e) & 1u)) {
          if constexpr (GB == 2) reinterpret_cast<uint16_t *>(g)[e] = 0;
          else reinterpret_cast<uint32_t *>(g)[e] = 0;
        }
      }
    }
  }
}

// Two bf16 gradients (one word) times t0 / t1, rounded to bf16, then (scale)
// times sb rounded again.  The hardware pair conversion rounds like
// f32_to_bf16_bits except for NaN (canonical NaN vs sign | 0x7FC0), so a
// pair holding a NaN takes the software rounding.
__device__ __forceinline__ uint32_t grad_pair(uint32_t gw, float t0, float t1, float sb,
                                              bool scale) {
  const float p0 = bf16_bits_to_f32(gw & 0xFFFFu) * t0;
  const float p1 = bf16_bits_to_f32(gw >> 16) * t1;
  uint32_t y = bf16x2_from_f32(p0, p1);
  const bool nan = (p0 != p0) | (p1 != p1);
  if (nan) y = f32_to_bf16_bits(p0) | (f32_to_bf16_bits(p1) << 16);
  if (!scale) return y;
  const float q0 = bf16_bits_to_f32(y & 0xFFFFu) * sb;
  const float q1 = bf16_bits_to_f32(y >> 16) * sb;
  if (nan | (q0 != q0) | (q1 != q1)) return f32_to_bf16_bits(q0) | (f32_to_bf16_bits(q1) << 16);
  return bf16x2_from_f32(q0, q1);
}

// grad <- bit ? bf16(grad * (2 k r)) : 0, then (SCALE) bf16(grad * bf16(scale)).
template <int SDT, bool PACK, bool SCALE>
__global__ void __launch_bounds__(kThreads) relu2_grad_kernel(const UnpackParams P) {
  using G = Chunk<2>;
  __shared__ __align__(16) uint8_t stage[kStageBytes];
  __shared__ uint32_t s_wt[G::S * 8];
  // fp8 storage: 2 k r depends on the 8-bit code alone -> a 256-entry table
  constexpr bool LUT = SDT != BS_BF16;
  __shared__ float lut[LUT ? 256 : 1];
  const int64_t pid0 = (int64_t)blockIdx.x * kUT;
  const int nt = tiles_here(P, pid0);
  const PidPos pp(pid0, P.grid_n);
  const int tid = threadIdx.x;
  const float two_k = 2.0f * P.k;
  if constexpr (LUT) lut[tid] = two_k * store_bits_to_f32<SDT>(tid);
  uint32_t m[G::S], cnt[G::S], ex[G::S];
#pragma unroll
  for (int s = 0; s < G::S; ++s) {  // masks first: independent of the values
    const int c = s * kThreads + tid;
    const int j = c / G::CPT, cc = c % G::CPT;
    m[s] = 0;
    if (j < nt) m[s] = load_mask<16>(P.bitmask + (pid0 + j) * kTileBytes + cc * 2);
  }
  const uint32_t first = stage_values<SDT, PACK>(P, pid0, nt, stage);
#pragma unroll
  for (int s = 0; s < G::S; ++s) cnt[s] = __popc(m[s]);
  block_excl_scan<G::S>(cnt, ex, s_wt);
  float sb = 0.f;
  if constexpr (SCALE) sb = bf16_bits_to_f32(f32_to_bf16_bits(*P.scale));
#pragma unroll
  for (int s = 0; s < G::S; ++s) {
    const int c = s * kThreads + tid;
    const int j = c / G::CPT, cc = c % G::CPT;
    if (j >= nt) continue;
    const int row = cc / G::CPR, colc = cc % G::CPR;
    int64_t tr, tc;
    pp.pos(j, tr, tc);
    const int64_t grow = tr * kTileM + row;
    const int64_t gcol = tc * kTileN + colc * 16;
    if (grow >= P.batch_rows) continue;
    uint16_t *g = reinterpret_cast<uint16_t *>(P.out + (grow * P.out_ld + gcol) * 2);
    const bool vec = P.out_v32 && gcol + 16 <= P.K;
    const uint32_t mm = m[s];
    uint32_t gw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (vec) {
      if (mm) ld_v8(g, gw);
    } else {
      for (int e = 0; e < 16; ++e)
        if (gcol + e < P.K) gw[e >> 1] |= (uint32_t)g[e] << (16 * (e & 1));
    }
    uint32_t o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint32_t r = ex[s];
    if constexpr (LUT && !PACK) {
      // branch-free: every element reads the code at its rank (the stage has
      // slack past the last value), pairs are rounded by the hardware
      // conversion and unset elements cleared afterwards
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t b0 = (mm >> (2 * i)) & 1u, b1 = (mm >> (2 * i + 1)) & 1u;
        const float t0 = lut[staged_value<SDT, PACK>(stage, first, r)];
        r += b0;
        const float t1 = lut[staged_value<SDT, PACK>(stage, first, r)];
        r += b1;
        const uint32_t keep = (0u - b0) & 0xFFFFu | ((0u - b1) & 0xFFFF0000u);
        o[i] = grad_pair(gw[i], t0, t1, sb, SCALE) & keep;
      }
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      if constexpr (LUT && !PACK) break;
      if (!((mm >> e) & 1u)) continue;
      const uint32_t code = staged_value<SDT, PACK>(stage, first, r++);
      float tk;
      if constexpr (LUT) tk = lut[code];
      else tk = two_k * store_bits_to_f32<SDT>(code);
      const uint32_t gb = (gw[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
      uint32_t y = f32_to_bf16_bits(bf16_bits_to_f32(gb) * tk);
      if constexpr (SCALE) y = f32_to_bf16_bits(bf16_bits_to_f32(y) * sb);
      o[e >> 1] |= y << (16 * (e & 1));
    }
    if (vec) {
      st_v8(g, o);
    } else {
      for (int e = 0; e < 16; ++e)
        if (gcol + e < P.K) g[e] = (uint16_t)(o[e >> 1] >> (16 * (e & 1)));
    }
  }
}


// Sparse chunk of the persistent reconstruct: the chunk's values (ranks r,
// r + 1, ... in the stage) scattered by their set bits into this thread's
// zeroed 32-byte row of `scratch` and written out with one 32-byte store
// (element stores at the right edge).  `trips`: the largest count of any
// lane of the warp (the loop runs in step across the warp).
template <int SDT, bool PACK, bool SQ = false>
__device__ __forceinline__ void scatter_chunk(const uint8_t *stg, uint32_t first, uint32_t r,
                                           uint32_t mm, uint32_t trips, uint8_t *scratch,
                                           uint8_t *dst, bool vec, int valid) {
  constexpr int SB = Elt<SDT>::bytes;
  constexpr int VEC = 32 / SB;
  const int tid = threadIdx.x;
  // the row's two 16-byte halves lie 512 bytes apart inside the warp's
  // kilobyte, so the zeroing stores and read-back loads of a warp touch
  // consecutive 16-byte words (no bank conflicts)
  uint8_t *h0 = scratch + (tid >> 5) * 1024 + (tid & 31) * 16;
  uint4 *q0 = reinterpret_cast<uint4 *>(h0), *q1 = reinterpret_cast<uint4 *>(h0 + 512);
  *q0 = make_uint4(0, 0, 0, 0);
  *q1 = make_uint4(0, 0, 0, 0);
  uint32_t left = mm;
  for (uint32_t k = 0; k < trips; ++k) {
    if (left) {
      const int e = __ffs(left) - 1;
      left &= left - 1;
      const uint32_t v = staged_value<SDT, PACK>(stg, first, r++);
      const int byte = e * SB;
      uint8_t *d = h0 + byte + (byte >= 16 ? 512 - 16 : 0);
      if constexpr (SB == 1) *d = (uint8_t)v;
      else *reinterpret_cast<uint16_t *>(d) = (uint16_t)v;
    }
  }
  const uint4 lo = *q0, hi = *q1;
  uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  if constexpr (SQ) {  // ReLU^2 of bf16 storage, k = 1: bf16(v * v)
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = bf16x2_mul(w[i], w[i]);
  }
  if (vec) {
    st_v8(dst, w);
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) {  // static indices keep w[] in registers
      if (e >= valid) break;
      if constexpr (SB == 1) dst[e] = (w[e >> 2] >> (8 * (e & 3))) & 0xFFu;
      else reinterpret_cast<uint16_t *>(dst)[e] = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
    }
  }
}

// Plain reconstruct (OUT 0), persistent and double-buffered.  CTA b takes
// tile pairs b, b + G, ...; while it expands one pair, the bulk-copy engine
// already brings the next pair's bitmask (1 KB) and value segment into the
// other buffer, and thread 0 holds the prefix pair for the one after that
// in registers -- the load chain (prefix -> values) that a short-lived CTA
// waits through is off the critical path.  Raw and packed storage; vals
// must be 16-byte aligned (the aligned 16-byte superset of a segment is
// copied, as the per-CTA kernel's vector loads read it).
constexpr int kPipeMaskBytes = kUT * kTileBytes;

// Status word of the reconstruct kernels (bs_unpack has no status argument):
// BS_STATUS_TIMEOUT when a bounded wait gave up.  Read with bs_unpack_status.
__device__ int32_t g_unpack_status = 0;

// SQ: the ReLU^2 reconstruct of bf16 storage with k = 1 (RELU2_SCALE): each
// output word squared with one bf16x2 product, the rounding of the
// reference's bf16 `v * v` (triton_kernels.py:238).
template <int SDT, bool PACK, bool SQ = false>
__global__ void __launch_bounds__(kThreads) unpack_pipe_kernel(const UnpackParams P) {
  static_assert(!SQ || SDT == BS_BF16, "the fused square is for bf16 storage");
  constexpr int SB = Elt<SDT>::bytes;
  using G = Chunk<SB>;
  __shared__ __align__(128) uint8_t stage[2][kStageBytes];
  __shared__ __align__(128) uint8_t mbuf[2][kPipeMaskBytes];
  __shared__ uint32_t s_wt[G::S * 8];
  __shared__ uint32_t s_first[2];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ __align__(16) uint8_t scratch[kThreads * 32];  // a 32-byte row per thread
  const int tid = threadIdx.x;
  const int64_t npairs = (P.ntiles + kUT - 1) / kUT;
  const int64_t G_ = gridDim.x;

  // thread 0: issue the copies of pair g into buffer `buf` (prefixes p0, p1)
  const int64_t voff = (tid == 0 && P.vals_offset) ? *P.vals_offset : 0;
  auto issue = [&](int64_t g, int buf, uint32_t p0, uint32_t p1) {
    const int64_t t0 = g * kUT;
    const int nt = (int)(P.ntiles - t0 < kUT ? P.ntiles - t0 : kUT);
    uint32_t cnt = p1 - p0;
    if (cnt > (uint32_t)(nt * kTileNumel)) cnt = nt * kTileNumel;
    const int64_t base = (int64_t)p0 + voff;
    int64_t a0, a1;
    uint32_t first;
    if constexpr (!PACK) {
      const int64_t b0 = base * SB;
      a0 = b0 & ~(int64_t)15;
      a1 = (b0 + (int64_t)cnt * SB + 15) & ~(int64_t)15;
      first = (uint32_t)((b0 - a0) / SB);
    } else {
      constexpr int B = pack_bits<SDT>();
      const int64_t bit0 = base * B;
      a0 = (bit0 >> 3) & ~(int64_t)15;
      a1 = ((((base + cnt) * B + 7) >> 3) + 15) & ~(int64_t)15;
      first = (uint32_t)(bit0 - a0 * 8);
    }
    const uint32_t vbytes = cnt ? (uint32_t)(a1 - a0) : 0u;
    const uint32_t mbytes = (uint32_t)(nt * kTileBytes);
    s_first[buf] = first;
    mbar_expect_tx(&bars[buf], mbytes + vbytes);
    bulk_load(mbuf[buf], P.bitmask + (P.first_tile + t0) * kTileBytes, mbytes, &bars[buf]);
    if (vbytes) bulk_load(stage[buf], P.vals + a0, vbytes, &bars[buf]);
  };
  auto prefix_pair = [&](int64_t g, uint32_t &p0, uint32_t &p1) {
    const int64_t t0 = g * kUT;
    const int nt = (int)(P.ntiles - t0 < kUT ? P.ntiles - t0 : kUT);
    p0 = P.prefix[P.first_tile + t0];
    p1 = P.prefix[P.first_tile + t0 + nt];
  };

  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  uint32_t np0 = 0, np1 = 0;  // thread 0: prefixes of the pair after the one in flight
  if (tid == 0 && blockIdx.x < npairs) {
    uint32_t p0, p1;
    prefix_pair(blockIdx.x, p0, p1);
    issue(blockIdx.x, 0, p0, p1);
    if (blockIdx.x + G_ < npairs) prefix_pair(blockIdx.x + G_, np0, np1);
  }
  for (int64_t it = 0;; ++it) {
    const int64_t g = blockIdx.x + it * G_;
    if (g >= npairs) break;
    const int buf = (int)(it & 1);
    if (tid == 0 && g + G_ < npairs) {
      issue(g + G_, buf ^ 1, np0, np1);
      if (g + 2 * G_ < npairs) prefix_pair(g + 2 * G_, np0, np1);
    }
    {
      bool ok = false;
      for (uint32_t n = 0; n < kMaxPolls && !(ok = mbar_try_wait(&bars[buf], (uint32_t)((it >> 1) & 1))); ++n) {
      }
      if (!ok && tid == 0) status_or(&g_unpack_status, BS_STATUS_TIMEOUT);
    }
    const int64_t pid0 = g * kUT;
    const int nt = tiles_here(P, pid0);
    const PidPos pp(pid0, P.grid_n);
    uint32_t m[G::S], cnt[G::S], ex[G::S];
#pragma unroll
    for (int s = 0; s < G::S; ++s) {
      const int c = s * kThreads + tid;
      const int j = c / G::CPT, cc = c % G::CPT;
      m[s] = j < nt ? load_mask<G::VEC>(mbuf[buf] + j * kTileBytes + cc * (G::VEC / 8)) : 0u;
      cnt[s] = __popc(m[s]);
    }
    block_excl_scan<G::S>(cnt, ex, s_wt);
    // Warp-uniform choice per slot: when no chunk of the warp holds more
    // than a quarter of its elements, each lane scatters only its chunk's
    // values into its own zeroed 32-byte row of shared scratch (a loop over
    // the set bits, as many trips as the fullest lane of the warp needs) and
    // writes the row out with one 32-byte store -- the cost follows the number
    // of values, not of elements.  Otherwise every element reads the value at
    // its rank (branch-free).
    uint32_t most = 0;
#pragma unroll
    for (int s = 0; s < G::S; ++s) most = max(most, __reduce_max_sync(0xFFFFFFFFu, cnt[s]));
    const uint8_t *stg = stage[buf];
    const uint32_t first = s_first[buf];
    if (most <= P.scatter_max) {
#pragma unroll
      for (int s = 0; s < G::S; ++s) {
        const int c = s * kThreads + tid;
        const int j = c / G::CPT, cc = c % G::CPT;
        if (j >= nt) continue;
        const int row = cc / G::CPR, colc = cc % G::CPR;
        int64_t tr, tc;
        pp.pos(j, tr, tc);
        const int64_t grow = tr * kTileM + row;
        const int64_t gcol = tc * kTileN + colc * G::VEC;
        if (grow >= P.batch_rows) continue;
        scatter_chunk<SDT, PACK, SQ>(stg, first, ex[s], m[s], most, scratch,
                                 P.out + (grow * P.out_ld + gcol) * SB,
                                 P.out_v32 && gcol + G::VEC <= P.K, (int)(P.K - gcol));
      }
    } else {
#pragma unroll
    for (int s = 0; s < G::S; ++s) {
      const int c = s * kThreads + tid;
      const int j = c / G::CPT, cc = c % G::CPT;
      if (j >= nt) continue;
      const int row = cc / G::CPR, colc = cc % G::CPR;
      int64_t tr, tc;
      pp.pos(j, tr, tc);
      const int64_t grow = tr * kTileM + row;
      const int64_t gcol = tc * kTileN + colc * G::VEC;
      if (grow >= P.batch_rows) continue;
      uint8_t *dst = P.out + (grow * P.out_ld + gcol) * SB;
      const uint32_t mm = m[s];
      uint32_t r = ex[s];
      uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if constexpr (!PACK && SB == 2) {
        // two elements per output word, joined by one byte permute
#pragma unroll
        for (int e = 0; e < G::VEC; e += 2) {
          const uint32_t b0 = (mm >> e) & 1u, b1 = (mm >> (e + 1)) & 1u;
          const uint32_t v0 = staged_value<SDT, PACK>(stg, first, r) & (0u - b0);
          r += b0;
          const uint32_t v1 = staged_value<SDT, PACK>(stg, first, r) & (0u - b1);
          r += b1;
          w[e >> 1] = __byte_perm(v0, v1, 0x5410);
        }
      } else
#pragma unroll
      for (int e = 0; e < G::VEC; ++e) {
        uint32_t v;
        if constexpr (!PACK) {
          // branch-free: read the value at this element's rank (the stage
          // has slack past the last value), keep it only if its bit is set
          const uint32_t bit = (mm >> e) & 1u;
          v = staged_value<SDT, PACK>(stg, first, r) & (0u - bit);
          r += bit;
        } else {
          if (!((mm >> e) & 1u)) continue;
          v = staged_value<SDT, PACK>(stg, first, r++);
        }
        if constexpr (SB == 1) w[e >> 2] |= v << (8 * (e & 3));
        else w[e >> 1] |= v << (16 * (e & 1));
      }
      if constexpr (SQ) {
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = bf16x2_mul(w[i], w[i]);
      }
      if (P.out_v32 && gcol + G::VEC <= P.K) {
        st_v8(dst, w);
      } else {
        for (int e = 0; e < G::VEC; ++e) {
          if (gcol + e >= P.K) break;
          if constexpr (SB == 1) dst[e] = (w[e >> 2] >> (8 * (e & 3))) & 0xFFu;
          else reinterpret_cast<uint16_t *>(dst)[e] = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
        }
      }
    }
    }
    fence_proxy_async_smem();  // this pair's buffer reads precede its next bulk copies
    __syncthreads();
  }
}

}  // namespace bs

using namespace bs;

namespace {

int launch_err() { return cudaGetLastError() == cudaSuccess ? BS_OK : BS_ERR_LAUNCH; }
bool aligned(const void *p, int a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
unsigned ctas(int64_t ntiles) { return (unsigned)((ntiles + kUT - 1) / kUT); }

// Resident CTAs of the pipelined kernel on the current device (cached).
template <int SDT, bool PACK, bool SQ = false>
int pipe_resident() {
  constexpr int kMaxDev = 64;
  static int cache[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 0;
  if (!cache[dev]) {
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, unpack_pipe_kernel<SDT, PACK, SQ>,
                                                      kThreads, 0) != cudaSuccess)
      return 0;
    cache[dev] = sms * per_sm;  // benign race: every writer stores the same value
  }
  return cache[dev];
}

template <int SDT, bool PACK>
int unpack_disp2(const UnpackParams &P, int relu2, bool scale, cudaStream_t st) {
  const dim3 g(ctas(P.ntiles));
  if (!relu2 && P.vals_v16 && aligned(P.bitmask, 16) && !getenv("BS_UNPACK_PER_CTA")) {
    const int res = pipe_resident<SDT, PACK>();
    const int64_t npairs = (P.ntiles + kUT - 1) / kUT;
    if (res > 0) {
      unpack_pipe_kernel<SDT, PACK>
          <<<(unsigned)(npairs < res ? npairs : res), kThreads, 0, st>>>(P);
      return launch_err();
    }
  }
  if constexpr (SDT == BS_BF16) {  // ReLU^2 of bf16 storage (k = 1, no scale): pipelined too
    if (relu2 && !scale && P.k == 1.0f && P.vals_v16 && aligned(P.bitmask, 16) &&
        !getenv("BS_UNPACK_PER_CTA")) {
      const int res = pipe_resident<SDT, PACK, true>();
      const int64_t npairs = (P.ntiles + kUT - 1) / kUT;
      if (res > 0) {
        unpack_pipe_kernel<SDT, PACK, true>
            <<<(unsigned)(npairs < res ? npairs : res), kThreads, 0, st>>>(P);
        return launch_err();
      }
    }
  }
  if (!relu2) unpack_kernel<SDT, PACK, 0, false><<<g, kThreads, 0, st>>>(P);
  else if (scale) unpack_kernel<SDT, PACK, 1, true><<<g, kThreads, 0, st>>>(P);
  else unpack_kernel<SDT, PACK, 1, false><<<g, kThreads, 0, st>>>(P);
  return launch_err();
}

template <int SDT>
int unpack_disp(const UnpackParams &P, int pack, int relu2, bool scale, cudaStream_t st) {
  return pack ? unpack_disp2<SDT, true>(P, relu2, scale, st)
              : unpack_disp2<SDT, false>(P, relu2, scale, st);
}

template <int SDT, bool PACK>
int relu2g_disp2(const UnpackParams &P, bool scale, cudaStream_t st) {
  const dim3 g(ctas(P.ntiles));
  if (scale) relu2_grad_kernel<SDT, PACK, true><<<g, kThreads, 0, st>>>(P);
  else relu2_grad_kernel<SDT, PACK, false><<<g, kThreads, 0, st>>>(P);
  return launch_err();
}

template <int SDT>
int relu2g_disp(const UnpackParams &P, int pack, bool scale, cudaStream_t st) {
  return pack ? relu2g_disp2<SDT, true>(P, scale, st) : relu2g_disp2<SDT, false>(P, scale, st);
}

bool store_dtype_ok(int dt) { return dt == BS_BF16 || dt == BS_E4M3 || dt == BS_E5M2; }

}  // namespace

extern "C" int bs_unpack(const void *vals, const uint8_t *bitmask, const uint32_t *prefix,
                         const int64_t *vals_offset, int store_dtype, int pack_sbit, void *out,
                         int64_t out_ld, int64_t first_m_tile, int64_t grid_n, int64_t K,
                         int64_t batch_rows, int64_t num_tiles_in_batch, int relu2,
                         const float *scale, void *stream) {
  if (!store_dtype_ok(store_dtype)) return BS_ERR_DTYPE;
  if (num_tiles_in_batch < 0 || first_m_tile < 0 || grid_n < 0 || K < 0 || batch_rows < 0 ||
      out_ld < K)
    return BS_ERR_SHAPE;
  if (num_tiles_in_batch == 0) return BS_OK;
  if (grid_n == 0 || num_tiles_in_batch > ((int64_t)1 << 31)) return BS_ERR_SHAPE;
  if (!bitmask || !prefix || !out) return BS_ERR_ARG;
  if (pack_sbit && !aligned(vals, 4)) return BS_ERR_ALIGN;
  if (!relu2 && scale) return BS_ERR_ARG;
  UnpackParams P{};
  P.vals = static_cast<const uint8_t *>(vals);
  P.bitmask = bitmask;
  P.prefix = prefix;
  P.vals_offset = vals_offset;
  P.out = static_cast<uint8_t *>(out);
  P.out_ld = out_ld;
  P.first_tile = first_m_tile * grid_n;
  P.ntiles = num_tiles_in_batch;
  P.grid_n = grid_n;
  P.K = K;
  P.batch_rows = batch_rows;
  P.scale = scale;
  P.k = 1.0f;
  const int ob = relu2 ? 2 : (store_dtype == BS_BF16 ? 2 : 1);
  P.vals_v16 = aligned(vals, 16);
  P.out_v32 = aligned(out, 32) && ((out_ld * ob) % 32 == 0);
  {  // a quarter of a 32-byte chunk's elements: measured on 8192 x 14336 bf16,
     // a larger limit is slower at 70% sparsity (half a chunk: 81.6 vs 74.0 us)
     // and gains nothing at 90% (72 us either way); BS_UNPACK_SCATTER_MAX
     // overrides it for measurements
    const char *e = getenv("BS_UNPACK_SCATTER_MAX");
    const int env_max = e ? atoi(e) : -1;
    P.scatter_max = env_max >= 0 ? (uint32_t)env_max : (uint32_t)(8 / ob);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (store_dtype) {
    case BS_BF16: return unpack_disp<BS_BF16>(P, pack_sbit, relu2, scale, st);
    case BS_E4M3: return unpack_disp<BS_E4M3>(P, pack_sbit, relu2, scale, st);
    default: return unpack_disp<BS_E5M2>(P, pack_sbit, relu2, scale, st);
  }
}

extern "C" int bs_unpack_tile_scaled(const void *vals, const uint8_t *bitmask,
                                     const uint32_t *prefix, const int64_t *vals_offset,
                                     int pack_sbit, const float *tile_scales, void *out,
                                     int64_t out_ld, int64_t first_m_tile, int64_t grid_n,
                                     int64_t K, int64_t batch_rows, int64_t num_tiles_in_batch,
                                     void *stream) {
  if (num_tiles_in_batch < 0 || first_m_tile < 0 || grid_n < 0 || K < 0 || batch_rows < 0 ||
      out_ld < K)
    return BS_ERR_SHAPE;
  if (num_tiles_in_batch == 0) return BS_OK;
  if (grid_n == 0 || num_tiles_in_batch > ((int64_t)1 << 31)) return BS_ERR_SHAPE;
  if (!bitmask || !prefix || !out || !tile_scales) return BS_ERR_ARG;
  if (pack_sbit && !aligned(vals, 4)) return BS_ERR_ALIGN;
  UnpackParams P{};
  P.vals = static_cast<const uint8_t *>(vals);
  P.bitmask = bitmask;
  P.prefix = prefix;
  P.vals_offset = vals_offset;
  P.out = static_cast<uint8_t *>(out);
  P.out_ld = out_ld;
  P.first_tile = first_m_tile * grid_n;
  P.ntiles = num_tiles_in_batch;
  P.grid_n = grid_n;
  P.K = K;
  P.batch_rows = batch_rows;
  P.tile_scales = tile_scales;
  P.vals_v16 = aligned(vals, 16);
  P.out_v32 = aligned(out, 32) && ((out_ld * 2) % 32 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 g(ctas(P.ntiles));
  if (pack_sbit) unpack_kernel<BS_E4M3, true, 3, false><<<g, kThreads, 0, st>>>(P);
  else unpack_kernel<BS_E4M3, false, 3, false><<<g, kThreads, 0, st>>>(P);
  return launch_err();
}

extern "C" int bs_mask_with_bitmask(void *grad, int grad_dtype, int64_t M, int64_t N,
                                    int64_t ld, const uint8_t *bitmask, void *stream) {
  if (grad_dtype != BS_BF16 && grad_dtype != BS_F32) return BS_ERR_DTYPE;
  if (M < 0 || N < 0 || ld < N) return BS_ERR_SHAPE;
  const int64_t gm = (M + 63) / 64, gn = (N + 63) / 64;
  if (gm * gn == 0) return BS_OK;
  if (gm * gn > ((int64_t)1 << 31)) return BS_ERR_SHAPE;
  if (!grad || !bitmask) return BS_ERR_ARG;
  UnpackParams P{};
  P.bitmask = bitmask;
  P.out = static_cast<uint8_t *>(grad);
  P.out_ld = ld;
  P.ntiles = gm * gn;
  P.grid_n = gn;
  P.K = N;
  P.batch_rows = M;
  const int gb = grad_dtype == BS_BF16 ? 2 : 4;
  P.out_v32 = aligned(grad, 32) && ((ld * gb) % 32 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (gb == 2) mask_kernel<2><<<ctas(P.ntiles), kThreads, 0, st>>>(P);
  else mask_kernel<4><<<ctas(P.ntiles), kThreads, 0, st>>>(P);
  return launch_err();
}

extern "C" int bs_relu2_grad(void *grad, int grad_dtype, int64_t M, int64_t N, int64_t ld,
                             const void *vals, const uint8_t *bitmask, const uint32_t *prefix,
                             const int64_t *vals_offset, int store_dtype, int pack_sbit,
                             const float *scale, void *stream) {
  if (grad_dtype != BS_BF16) return BS_ERR_DTYPE;
  if (!store_dtype_ok(store_dtype)) return BS_ERR_DTYPE;
  if (M < 0 || N < 0 || ld < N) return BS_ERR_SHAPE;
  const int64_t gm = (M + 63) / 64, gn = (N + 63) / 64;
  if (gm * gn == 0) return BS_OK;
  if (gm * gn > ((int64_t)1 << 31)) return BS_ERR_SHAPE;
  if (!grad || !bitmask || !prefix) return BS_ERR_ARG;
  if (pack_sbit && !aligned(vals, 4)) return BS_ERR_ALIGN;
  UnpackParams P{};
  P.vals = static_cast<const uint8_t *>(vals);
  P.bitmask = bitmask;
  P.prefix = prefix;
  P.vals_offset = vals_offset;
  P.out = static_cast<uint8_t *>(grad);
  P.out_ld = ld;
  P.ntiles = gm * gn;
  P.grid_n = gn;
  P.K = N;
  P.batch_rows = M;
  P.scale = scale;
  P.k = 1.0f;
  P.vals_v16 = aligned(vals, 16);
  P.out_v32 = aligned(grad, 32) && ((ld * 2) % 32 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool sc = scale != nullptr;
  switch (store_dtype) {
    case BS_BF16: return relu2g_disp<BS_BF16>(P, pack_sbit, sc, st);
    case BS_E4M3: return relu2g_disp<BS_E4M3>(P, pack_sbit, sc, st);
    default: return relu2g_disp<BS_E5M2>(P, pack_sbit, sc, st);
  }
}

namespace bs {
namespace {

// Largest stored code of one tensor's raw fp8 values [off, off + nnz): the
// stored values are positive, so the largest code is the largest value.
__global__ void __launch_bounds__(kThreads)
code_max_kernel(const uint8_t *vals, const int64_t *vals_offset, const uint32_t *prefix_last,
                uint32_t *out) {
  const int64_t off = vals_offset ? *vals_offset : 0;
  const int64_t n = *prefix_last;
  const uint8_t *p = vals + off;
  // bytes before the first 16-byte boundary and after the last one singly,
  // the aligned body as 16-byte vectors with a byte-wise max
  const int64_t h16 = (int64_t)((16 - (reinterpret_cast<uintptr_t>(p) & 15)) & 15);
  const int64_t head = n < h16 ? n : h16;
  const int64_t nv = (n - head) / 16;
  const int64_t tail0 = head + nv * 16;
  const int64_t gid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  uint32_t m4 = 0;
  const uint4 *pv = reinterpret_cast<const uint4 *>(p + head);
  for (int64_t i = gid; i < nv; i += stride) {
    const uint4 v = ld_nc_v4(pv + i);
    m4 = __vmaxu4(m4, __vmaxu4(__vmaxu4(v.x, v.y), __vmaxu4(v.z, v.w)) & 0x7F7F7F7Fu);
  }
  if (gid < head) m4 = __vmaxu4(m4, p[gid] & 0x7Fu);
  if (gid < n - tail0) m4 = __vmaxu4(m4, p[tail0 + gid] & 0x7Fu);
  uint32_t m = max(max(m4 & 0xFFu, (m4 >> 8) & 0xFFu), max((m4 >> 16) & 0xFFu, m4 >> 24));
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, d));
  if ((threadIdx.x & 31) == 0 && m) atomicMax(out, m);
}

// to_fp8 scale of the ReLU^2 reconstruction k x^2 (x fp8 as fp32, rounded
// to bf16, then times bf16(scale^2) rounded to bf16): it is non-decreasing
// in x >= 0, so its amax is its value at the largest stored code.  Resets
// the scratch word.
template <int SDT>
__global__ void relu2_qscale_kernel(uint32_t *code_ws, const float *scale, float k,
                                    float *qscale, int compiled) {
  const float x = store_bits_to_f32<SDT>(*code_ws);
  float v = bf16_bits_to_f32(f32_to_bf16_bits(k * x * x));
  if (scale) {
    const float sc = *scale;
    v = bf16_bits_to_f32(f32_to_bf16_bits(v * bf16_bits_to_f32(f32_to_bf16_bits(sc * sc))));
  }
  float s = compiled ? v * kRcp448 : __fdiv_rn(v, 448.0f);
  if (!compiled) s = bf16_bits_to_f32(f32_to_bf16_bits(s));
  *qscale = fmaxf(s, 1e-9f);
  *code_ws = 0u;
}

}  // namespace
}  // namespace bs

extern "C" int bs_unpack_relu2_fp8t(const void *vals, const uint8_t *bitmask,
                                    const uint32_t *prefix, const int64_t *vals_offset,
                                    int store_dtype, int64_t M, int64_t N, const float *scale,
                                    float k, uint32_t *code_ws, float *qscale_out, void *outT,
                                    int64_t out_ld, int fp8_flags, void *stream) {
  const int compiled = (fp8_flags & BS_FP8_COMPILED) != 0;
  if (store_dtype != BS_E4M3 && store_dtype != BS_E5M2) return BS_ERR_DTYPE;
  if (M < 0 || N < 0 || out_ld < M) return BS_ERR_SHAPE;
  const int64_t gm = (M + kTileM - 1) / kTileM, gn = (N + kTileN - 1) / kTileN;
  if (!bitmask || !prefix || !code_ws || !qscale_out || (gm * gn && !outT)) return BS_ERR_ARG;
  if (gm * gn > ((int64_t)1 << 31)) return BS_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t *v8 = static_cast<const uint8_t *>(vals);
  code_max_kernel<<<148 * 4, kThreads, 0, st>>>(v8, vals_offset, prefix + gm * gn, code_ws);
  if (store_dtype == BS_E4M3)
    relu2_qscale_kernel<BS_E4M3><<<1, 1, 0, st>>>(code_ws, scale, k, qscale_out, compiled);
  else
    relu2_qscale_kernel<BS_E5M2><<<1, 1, 0, st>>>(code_ws, scale, k, qscale_out, compiled);
  if (gm * gn == 0) return launch_err();
  UnpackParams P{};
  P.vals = v8;
  P.bitmask = bitmask;
  P.prefix = prefix;
  P.vals_offset = vals_offset;
  P.out = static_cast<uint8_t *>(outT);
  P.out_ld = out_ld;
  P.first_tile = 0;
  P.ntiles = gm * gn;
  P.grid_n = gn;
  P.K = N;
  P.batch_rows = M;
  P.scale = scale;
  P.k = k;
  P.qscale = qscale_out;
  P.qcompiled = compiled;
  P.vals_v16 = aligned(vals, 16);
  P.out_v32 = aligned(outT, 16) && (out_ld % 16 == 0);
  const dim3 g(ctas(P.ntiles));
  if (store_dtype == BS_E4M3) {
    if (scale) unpack_kernel<BS_E4M3, false, 2, true><<<g, kThreads, 0, st>>>(P);
    else unpack_kernel<BS_E4M3, false, 2, false><<<g, kThreads, 0, st>>>(P);
  } else {
    if (scale) unpack_kernel<BS_E5M2, false, 2, true><<<g, kThreads, 0, st>>>(P);
    else unpack_kernel<BS_E5M2, false, 2, false><<<g, kThreads, 0, st>>>(P);
  }
  return launch_err();
}

extern "C" int bs_unpack_status(int32_t *status_out, int reset) {
  if (!status_out) return BS_ERR_ARG;
  // synchronous on the device: every reconstruct launched so far has finished
  if (cudaMemcpyFromSymbol(status_out, g_unpack_status, sizeof(int32_t)) != cudaSuccess)
    return BS_ERR_LAUNCH;
  if (reset && *status_out) {
    const int32_t zero = 0;
    if (cudaMemcpyToSymbol(g_unpack_status, &zero, sizeof(int32_t)) != cudaSuccess)
      return BS_ERR_LAUNCH;
  }
  return BS_OK;
}
