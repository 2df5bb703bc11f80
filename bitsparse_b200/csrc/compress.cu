// K1 -- fused compress: dense -> bitmask, prefix, compacted values.
//
// Reference behaviour replaced (Maxzhu123/bitsparse):
//   _tile_pack_kernel     lib_sparse/src/triton_kernels.py:63-97
//   torch.cumsum prefix   lib_sparse/src/functions.py:33-40
//   _compact_vals_kernel  lib_sparse/src/triton_kernels.py:105-146
//   _pack_kernel          lib_sparse/src/bitpacking.py:58-117
//   arena offset update   lib_sparse/src/functions.py:73-92
//
// Work decomposition.  A CTA of 256 threads owns a "partition" of TPP
// consecutive tiles (tile id order = output order).  Each thread owns 32-byte
// chunks (16 bf16 / 32 fp8 / 8 fp32 elements of one tile row), read with one
// 256-bit load; a warp covers whole tile rows, so every DRAM sector is used in
// full.  All of a thread's loads are issued before any is consumed.  A
// chunk's mask bits are exactly its 2 / 4 / 1 bitmask bytes in the
// reference's LSB-first, row-major-in-tile order; they are computed with SWAR
// integer arithmetic on the raw bits (x > 0 <=> 0 < bits <= +inf /
// max-finite).
//
// The fused compress (MODE 0) is two wait-free kernels:
//  1. count_kernel, partitions in order: loads the dense tiles from DRAM,
//     writes the bitmask bytes (and the dense e4m3 tensor when quantising),
//     stores the partition's nonzero count and adds it to its segment total
//     (a segment = 256 partitions); block 0 snapshots the TensorBuffer offset.
//  2. compact_kernel, partitions in REVERSE order: the partitions counted last
//     are still resident in the 126 MB L2, so a large share of this second
//     read never reaches DRAM.  While its loads are in flight, warp 0 sums the
//     preceding segment totals and the preceding counts of its own segment to
//     get the partition's base; the CTA reads its masks back from the bitmask,
//     scans them, writes the tile prefixes and the values.  The last
//     partition publishes the totals (arena offset, vals_offset, nnz).
// No CTA ever waits for another one; ordering comes from the stream.  An
// earlier single-kernel design with a decoupled look-back made every CTA
// wait on the slowest of the hundreds of partitions between it and the
// inclusive frontier and reached only ~20% of HBM bandwidth on B200.
//
// Values.  Raw storage: staged in shared memory already shifted by the
// destination's misalignment, then written with aligned 16-byte stores
// (element stores only for the two edge vectors shared with neighbouring
// partitions).  Packed storage (15/7-bit): re-packed into 32-bit words of the
// continuous bitstream; words shared with a neighbouring partition are merged
// with atomicAnd / atomicOr on disjoint bit masks (order independent).
#include "common.cuh"

#include <mutex>

namespace bs {

// Workspace: header {off0}, uint64 segment totals (zeroed by a memset before
// the count kernel), uint32 per-partition counts.
struct WsHeader {
  long long off0;  // logical index of this tensor's first value
  unsigned long long pad[15];
};
constexpr int kSeg = 256;  // partitions per segment

struct CompressParams {
  const uint8_t *dense;
  int64_t M, N, ld;
  const float *qscale;
  uint8_t *qout;
  uint8_t *bitmask;
  uint32_t *prefix;
  uint8_t *vals;
  int64_t cap;  // raw: elements, packed: bytes
  int64_t *arena_offset;
  int64_t *vals_offset_out;
  int64_t *nnz_out;
  int32_t *counts;  // MODE 2 only
  WsHeader *hdr;
  unsigned long long *seg_ws;  // MODE 0: per-segment totals
  uint32_t *counts_ws;         // MODE 0: per-partition counts
  int32_t *status;
  int64_t grid_n, num_tiles, num_parts;
  int vec_ok;    // dense base / row stride allow 32-byte vector loads
  int vals_v16;  // vals base 16-byte aligned (raw storage)
  int qout_vec;  // quant_out allows chunk-wide stores
};

template <int DT_IN, bool QUANT, int TPP>
struct Cfg {
  static constexpr int SDT = QUANT ? BS_E4M3 : DT_IN;  // stored dtype
  static constexpr int EB = Elt<DT_IN>::bytes;          // input bytes
  static constexpr int SB = Elt<SDT>::bytes;            // stored bytes
  static constexpr int VEC = 32 / EB;                   // elements per chunk
  static constexpr int CPR = kTileN / VEC;              // chunks per tile row
  static constexpr int CPT = kTileNumel / VEC;          // chunks per tile
  static constexpr int S = TPP * CPT / kThreads;        // chunk slots per thread
  static constexpr int SW = VEC * SB / 4;               // stored u32 words / chunk
  static constexpr int EPV = 16 / SB;                   // stored elts per 16 B
  static constexpr int BITS = pack_bits<SDT>();
  static_assert(TPP * CPT % kThreads == 0, "partition must fill whole slots");
};

// ---------------------------------------------------------------------------
// Positive masks on raw bits, one u32 word at a time.
// ---------------------------------------------------------------------------
// bf16 pair: bit 15 / bit 31 set iff that half is in (0, 0x7F80].
__device__ __forceinline__ uint32_t pos_bf16x2(uint32_t w) {
  const uint32_t v = w & 0x7FFF7FFFu;
  const uint32_t nz = v + 0x7FFF7FFFu;   // bit 15 of a half set iff v != 0
  const uint32_t nan = v + 0x007F007Fu;  // bit 15 set iff v >= 0x7F81 (NaN)
  return nz & ~nan & ~w & 0x80008000u;   // ~w: sign bit clear
}
// fp8 quad: bit 7 of a byte set iff the byte is in (0, LIM].
template <uint32_t LIM>
__device__ __forceinline__ uint32_t pos_fp8x4(uint32_t w) {
  const uint32_t v = w & 0x7F7F7F7Fu;
  const uint32_t nz = v + 0x7F7F7F7Fu;
  const uint32_t big = v + (0x7Fu - LIM) * 0x01010101u;  // bit 7 iff v > LIM
  return nz & ~big & ~w & 0x80808080u;
}
// Gather bit 7 of each byte of p into 4 consecutive bits (no carries: the
// 16 partial products land on distinct bit positions).
__device__ __forceinline__ uint32_t gather4(uint32_t p) {
  return (((p >> 7) * 0x00204081u) >> 21) & 0xFu;
}

template <int SDT, int NWORDS>
__device__ __forceinline__ uint32_t mask_of_words(const uint32_t *w) {
  uint32_t m = 0;
  if constexpr (SDT == BS_BF16) {
    uint32_t q = 0;
#pragma unroll
    for (int i = 0; i < NWORDS; ++i) q |= pos_bf16x2(w[i]) >> (15 - 2 * i);
    m = (q & 0x5555u) | ((q >> 15) & 0xAAAAu);
  } else {
    constexpr uint32_t LIM = SDT == BS_E4M3 ? 0x7Eu : 0x7Cu;
#pragma unroll
    for (int i = 0; i < NWORDS; ++i) m |= gather4(pos_fp8x4<LIM>(w[i])) << (4 * i);
  }
  return m;
}

// ---------------------------------------------------------------------------
// Chunks: load 32 B raw (issued early), then stored words + mask.
// ---------------------------------------------------------------------------
template <int EB>
__device__ __forceinline__ void load_raw(const CompressParams &P, int64_t grow, int64_t gcol,
                                         uint32_t (&raw)[8]) {
  constexpr int VEC = 32 / EB;
#pragma unroll
  for (int i = 0; i < 8; ++i) raw[i] = 0;
  if (grow >= P.M) return;
  const uint8_t *src = P.dense + (grow * P.ld + gcol) * EB;
  if (P.vec_ok && gcol + VEC <= P.N) {
    asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(raw[0]), "=r"(raw[1]), "=r"(raw[2]), "=r"(raw[3]), "=r"(raw[4]),
                   "=r"(raw[5]), "=r"(raw[6]), "=r"(raw[7])
                 : "l"(src));
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      if (gcol + e < P.N) {
        uint32_t b;
        if constexpr (EB == 1) b = src[e];
        else if constexpr (EB == 2) b = reinterpret_cast<const uint16_t *>(src)[e];
        else b = reinterpret_cast<const uint32_t *>(src)[e];
        raw[e * EB / 4] |= b << (8 * ((e * EB) & 3));
      }
    }
  }
}

// raw (in place) -> stored words (first SW words) + mask.  With QUANT the
// input is quantised to e4m3 as to_fp8 does; `side_outputs` also writes the
// dense e4m3 tensor.
template <int DT_IN, bool QUANT, int TPP>
__device__ __forceinline__ uint32_t process_chunk(const CompressParams &P, int64_t grow,
                                                  int64_t gcol, float qs, uint32_t (&raw)[8],
                                                  bool side_outputs) {
  using C = Cfg<DT_IN, QUANT, TPP>;
  if constexpr (!QUANT) {
    return mask_of_words<C::SDT, 8>(raw);
  } else {
    uint32_t sv[C::SW];
#pragma unroll
    for (int i = 0; i < C::SW; ++i) sv[i] = 0;
    if constexpr (DT_IN == BS_BF16) {
      // |x / scale| <= 448 * (1 + 2^-8): the fast paths are exact here
      const float r = __frcp_rn(qs);
#pragma unroll
      for (int e = 0; e < C::VEC; e += 2) {
        const float y0 = div_round_bf16(bf16_bits_to_f32((raw[e >> 1] & 0xFFFFu)), qs, r);
        const float y1 = div_round_bf16(bf16_bits_to_f32(raw[e >> 1] >> 16), qs, r);
        sv[e >> 2] |= e4m3x2_bits(y0, y1) << (8 * (e & 3));
      }
    } else {
#pragma unroll
      for (int e = 0; e < C::VEC; ++e) {
        const float y = __fdiv_rn(__uint_as_float(raw[e]), qs);
        sv[e >> 2] |= f32_to_e4m3_bits(y) << (8 * (e & 3));
      }
    }
    if (side_outputs && P.qout && grow < P.M) {
      uint8_t *dst = P.qout + grow * P.N + gcol;
      if (P.qout_vec && gcol + C::VEC <= P.N) {
        if constexpr (C::SW == 2) *reinterpret_cast<uint2 *>(dst) = make_uint2(sv[0], sv[1]);
        else *reinterpret_cast<uint4 *>(dst) = make_uint4(sv[0], sv[1], sv[2], sv[3]);
      } else {
#pragma unroll
        for (int e = 0; e < C::VEC; ++e)
          if (gcol + e < P.N) dst[e] = (sv[e >> 2] >> (8 * (e & 3))) & 0xFFu;
      }
    }
#pragma unroll
    for (int i = 0; i < C::SW; ++i) raw[i] = sv[i];
    return mask_of_words<BS_E4M3, C::SW>(sv);
  }
}

// Write the bits `own` of word *dst (other bits untouched).
__device__ __forceinline__ void merge_word(uint32_t *dst, uint32_t val, uint32_t own) {
  if (own == 0xFFFFFFFFu) {
    *dst = val;
  } else if (own) {
    atomicAnd(dst, ~own);
    atomicOr(dst, val & own);
  }
}

// Grid position of the TPP consecutive tiles of a partition: one 32-bit
// division per thread (num_tiles < 2^31), a bounded wrap per tile.
template <int TPP>
struct PartTiles {
  uint32_t tm0, tn0, gn;
  long long t0, nt;
  __device__ __forceinline__ PartTiles(const CompressParams &P, long long part) {
    gn = (uint32_t)P.grid_n;
    t0 = part * TPP;
    nt = P.num_tiles;
    tm0 = (uint32_t)t0 / gn;
    tn0 = (uint32_t)t0 - tm0 * gn;
  }
  __device__ __forceinline__ bool valid(int j) const { return t0 + j < nt; }
  __device__ __forceinline__ void pos(int j, uint32_t &tm, uint32_t &tn) const {
    tm = tm0;
    tn = tn0 + (uint32_t)j;
    while (tn >= gn) { tn -= gn; ++tm; }
  }
};

// Issue the loads of a partition (all slots), no use yet.
template <int DT_IN, bool QUANT, int TPP>
__device__ __forceinline__ void issue_partition(const CompressParams &P, const PartTiles<TPP> &pt,
                                                uint32_t (&raw)[Cfg<DT_IN, QUANT, TPP>::S][8]) {
  using C = Cfg<DT_IN, QUANT, TPP>;
#pragma unroll
  for (int s = 0; s < C::S; ++s) {
    const int c = s * kThreads + threadIdx.x;
    const int j = c / C::CPT, cc = c % C::CPT;
    const int row = cc / C::CPR, colc = cc % C::CPR;
    uint32_t tm, tn;
    pt.pos(j, tm, tn);
    // out-of-range tiles: a row past M loads nothing (zeros)
    load_raw<C::EB>(P, pt.valid(j) ? (int64_t)tm * kTileM + row : P.M,
                    (int64_t)tn * kTileN + colc * C::VEC, raw[s]);
  }
}

// Masks (+ bitmask bytes, + quantisation) of a loaded partition.  With
// MASK_FROM_BITMASK (raw storage) the masks are read back from the bitmask
// the counting pass wrote instead of being recomputed.
template <int DT_IN, bool QUANT, int TPP, bool WRITE_BITMASK, bool MASK_FROM_BITMASK = false>
__device__ __forceinline__ void process_partition(const CompressParams &P, long long part,
                                                  const PartTiles<TPP> &pt,
                                                  uint32_t (&raw)[Cfg<DT_IN, QUANT, TPP>::S][8],
                                                  uint32_t (&msk)[Cfg<DT_IN, QUANT, TPP>::S]) {
  using C = Cfg<DT_IN, QUANT, TPP>;
  const float qs = QUANT ? *P.qscale : 1.f;
#pragma unroll
  for (int s = 0; s < C::S; ++s) {
    const int c = s * kThreads + threadIdx.x;
    const int j = c / C::CPT, cc = c % C::CPT;
    const long long tile = part * TPP + j;
    msk[s] = 0;
    if (!pt.valid(j)) continue;
    uint8_t *bm = P.bitmask + tile * kTileBytes + cc * (C::VEC / 8);
    if constexpr (MASK_FROM_BITMASK && !QUANT) {
      if constexpr (C::VEC == 8) msk[s] = *bm;
      else if constexpr (C::VEC == 16) msk[s] = *reinterpret_cast<const uint16_t *>(bm);
      else msk[s] = *reinterpret_cast<const uint32_t *>(bm);
    } else {
      const int row = cc / C::CPR, colc = cc % C::CPR;
      uint32_t tm, tn;
      pt.pos(j, tm, tn);
      msk[s] = process_chunk<DT_IN, QUANT, TPP>(P, (int64_t)tm * kTileM + row,
                                                (int64_t)tn * kTileN + colc * C::VEC, qs,
                                                raw[s], WRITE_BITMASK);
      if (WRITE_BITMASK) {
        if constexpr (C::VEC == 8) *bm = (uint8_t)msk[s];
        else if constexpr (C::VEC == 16) *reinterpret_cast<uint16_t *>(bm) = (uint16_t)msk[s];
        else *reinterpret_cast<uint32_t *>(bm) = msk[s];
      }
    }
  }
}

// Block scan of chunk counts in (slot, warp, lane) order: per-thread
// exclusive offsets in `lex` + s_wt (exclusive per warp slot); returns the
// partition total and fills s_tile_incl (inclusive count after each tile).
template <typename C, int TPP>
__device__ __forceinline__ uint32_t partition_scan(const uint32_t (&msk)[C::S],
                                                   uint32_t (&lex)[C::S], uint32_t *s_wt,
                                                   uint32_t *s_tile_incl, uint32_t *s_total) {
  constexpr int NW = C::S * 8;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int s = 0; s < C::S; ++s) {
    const uint32_t cnt = __popc(msk[s]);
    const uint32_t inc = warp_incl_scan(cnt);
    lex[s] = inc - cnt;
    if (lane == 31) s_wt[s * 8 + warp] = inc;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t carry = 0;
#pragma unroll
    for (int w0 = 0; w0 < NW; w0 += 32) {
      const int idx = w0 + lane;
      const uint32_t v = idx < NW ? s_wt[idx] : 0;
      const uint32_t inc = warp_incl_scan(v) + carry;
      if (idx < NW) s_wt[idx] = inc - v;
      carry = __shfl_sync(0xFFFFFFFFu, inc, 31);
    }
    if (lane == 0) *s_total = carry;
  }
  __syncthreads();
  const uint32_t total = *s_total;
  if (tid < TPP) {
    const int nxt = (tid + 1) * C::CPT / 32;  // warp slot that starts tile tid+1
    s_tile_incl[tid] = nxt < NW ? s_wt[nxt] : total;
  }
  __syncthreads();
  return total;
}

// Stage a partition's values (chunk order) in shared memory and write them
// out.  `own_tail`: this partition owns (and zeroes) the packed stream after
// its payload up to packed_storage_nbytes(nnz) (standalone, last partition).
template <typename C, bool PACK>
__device__ __forceinline__ void write_values(const CompressParams &P, uint8_t *stage,
                                             const uint32_t (&msk)[C::S],
                                             const uint32_t (&sv)[C::S][8],
                                             const uint32_t (&lex)[C::S], const uint32_t *s_wt,
                                             long long gbase, long long n, bool own_tail) {
  const int tid = threadIdx.x, warp = tid >> 5;
  const int shift = PACK ? 0 : (int)(gbase % C::EPV);
#pragma unroll
  for (int s = 0; s < C::S; ++s) {
    const uint32_t m = msk[s];
    uint32_t k = shift + s_wt[s * 8 + warp] + lex[s];
#pragma unroll
    for (int e = 0; e < C::VEC; ++e) {  // static indices keep sv in registers
      if ((m >> e) & 1u) {
        if constexpr (C::SB == 1) {
          stage[k] = (uint8_t)(sv[s][e >> 2] >> (8 * (e & 3)));
        } else {
          reinterpret_cast<uint16_t *>(stage)[k] = (uint16_t)(sv[s][e >> 1] >> (16 * (e & 1)));
        }
        ++k;
      }
    }
  }
  __syncthreads();

  if constexpr (!PACK) {
    if (n == 0) return;
    const long long cap = P.cap;
    if (tid == 0 && gbase + n > cap) status_or(P.status, BS_STATUS_CAPACITY);
    const long long v0 = (gbase - shift) / C::EPV;
    const long long v1 = (gbase + n - 1) / C::EPV;
    for (long long v = v0 + tid; v <= v1; v += kThreads) {
      const long long e0 = v * C::EPV;
      const uint8_t *src = stage + (v - v0) * 16;
      if (P.vals_v16 && e0 >= gbase && e0 + C::EPV <= gbase + n && e0 + C::EPV <= cap) {
        st_v4(P.vals + e0 * C::SB, *reinterpret_cast<const uint4 *>(src));
      } else {
        for (int e = 0; e < C::EPV; ++e) {
          const long long g = e0 + e;
          if (g >= gbase && g < gbase + n && g < cap) {
            if constexpr (C::SB == 1) P.vals[g] = src[e];
            else reinterpret_cast<uint16_t *>(P.vals)[g] =
                reinterpret_cast<const uint16_t *>(src)[e];
          }
        }
      }
    }
  } else {
    constexpr int B = C::BITS;
    const long long bit0 = gbase * B;
    const long long bit1 = (gbase + n) * B;
    const long long cap_words = P.cap / 4;
    long long own_end = bit1;
    if (own_tail) {  // payload rounded to a word plus one guard word (bitpacking.py:32-34)
      const long long words = ((bit1 + 31) >> 5) + 1;
      own_end = (words < cap_words ? words : cap_words) * 32;
    }
    if (own_end <= bit0) return;
    const long long w0 = bit0 >> 5, w1 = (own_end - 1) >> 5;
    if (tid == 0 && ((bit1 + 31) >> 5) > cap_words) status_or(P.status, BS_STATUS_CAPACITY);
    uint32_t *words = reinterpret_cast<uint32_t *>(P.vals);
    for (long long w = w0 + tid; w <= w1; w += kThreads) {
      if (w >= cap_words) break;
      const long long wb = w * 32;
      unsigned long long acc = 0;
      const long long rel = wb - bit0;  // bit offset of the word inside our range
      for (long long k = rel > 0 ? rel / B : 0; k < n; ++k) {
        const long long sb = bit0 + k * B - wb;  // start of value k rel. to word
        if (sb >= 32) break;
        uint32_t v;
        if constexpr (C::SB == 1) v = stage[k];
        else v = reinterpret_cast<const uint16_t *>(stage)[k];
        acc |= (unsigned long long)(v & ((1u << B) - 1u)) << (sb + 32);  // sb > -B
      }
      const long long lo = bit0 > wb ? bit0 - wb : 0;
      const long long hi = own_end < wb + 32 ? own_end - wb : 32;
      const uint32_t own = (hi >= 32 ? 0xFFFFFFFFu : ((1u << hi) - 1u)) & ~((1u << lo) - 1u);
      merge_word(words + w, (uint32_t)(acc >> 32), own);
    }
  }
}

// ---------------------------------------------------------------------------
// MODE 1: compact only -- bases from a given prefix[] (the reference's
//         compact_vals); bitmask / prefix are not written.
// MODE 2: tile_pack only -- bitmask + per-tile counts, no values.
// ---------------------------------------------------------------------------
template <int DT_IN, bool QUANT, bool PACK, int TPP, int MODE>
__global__ void __launch_bounds__(kThreads) compress_kernel(const CompressParams P) {
  using C = Cfg<DT_IN, QUANT, TPP>;
  extern __shared__ __align__(128) uint8_t smem_dyn[];
  __shared__ uint32_t s_wt[C::S * 8];
  __shared__ uint32_t s_tile_incl[TPP];
  __shared__ uint32_t s_total;
  const long long part = blockIdx.x;
  uint32_t sv[C::S][8], msk[C::S], lex[C::S];
  const PartTiles<TPP> pt(P, part);
  issue_partition<DT_IN, QUANT, TPP>(P, pt, sv);
  process_partition<DT_IN, QUANT, TPP, MODE == 2>(P, part, pt, sv, msk);
  const uint32_t total = partition_scan<C, TPP>(msk, lex, s_wt, s_tile_incl, &s_total);
  const int tid = threadIdx.x;
  if (MODE == 2) {
    if (tid < TPP && part * TPP + tid < P.num_tiles)
      P.counts[part * TPP + tid] =
          (int32_t)(s_tile_incl[tid] - (tid ? s_tile_incl[tid - 1] : 0u));
    return;
  }
  const long long off = P.arena_offset ? *P.arena_offset : 0;  // vals_offset
  const long long gbase = off + (long long)P.prefix[part * TPP];
  write_values<C, PACK>(P, smem_dyn, msk, sv, lex, s_wt, gbase, total, false);
}

// ---------------------------------------------------------------------------
// MODE 0: count pass, then compact pass (see the file comment).
// ---------------------------------------------------------------------------
template <int DT_IN, bool QUANT, bool PACK, int TPP>
__global__ void __launch_bounds__(kThreads) count_kernel(const CompressParams P) {
  using C = Cfg<DT_IN, QUANT, TPP>;
  __shared__ uint32_t s_red[kThreads / 32];
  const long long part = blockIdx.x;
  uint32_t raw[C::S][8], msk[C::S];
  const PartTiles<TPP> pt(P, part);
  issue_partition<DT_IN, QUANT, TPP>(P, pt, raw);
  process_partition<DT_IN, QUANT, TPP, true>(P, part, pt, raw, msk);
  uint32_t c = 0;
#pragma unroll
  for (int s = 0; s < C::S; ++s) c += __popc(msk[s]);
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, d);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) s_red[warp] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) t += s_red[i];
    P.counts_ws[part] = t;
    atomicAdd(&P.seg_ws[part / kSeg], (unsigned long long)t);
    if (part == 0) {
      long long off = 0;
      if (P.arena_offset) {
        off = *P.arena_offset;
        if (PACK) off = (off + 7) / 8 * 8;  // functions.py:78-81
      }
      P.hdr->off0 = off;
    }
  }
}

template <int DT_IN, bool QUANT, bool PACK, int TPP>
__global__ void __launch_bounds__(kThreads) compact_kernel(const CompressParams P) {
  using C = Cfg<DT_IN, QUANT, TPP>;
  extern __shared__ __align__(128) uint8_t smem_dyn[];
  __shared__ uint32_t s_wt[C::S * 8];
  __shared__ uint32_t s_tile_incl[TPP];
  __shared__ uint32_t s_total;
  __shared__ long long s_excl;
  const long long part = P.num_parts - 1 - blockIdx.x;  // reverse: L2-resident first
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t raw[C::S][8], msk[C::S], lex[C::S];
  const PartTiles<TPP> pt(P, part);
  issue_partition<DT_IN, QUANT, TPP>(P, pt, raw);
  if (warp == 0) {  // this partition's base, while the loads are in flight
    const long long sg = part / kSeg;
    unsigned long long sum = 0;
    for (long long i = lane; i < sg; i += 32) sum += P.seg_ws[i];
    for (long long i = sg * kSeg + lane; i < part; i += 32) sum += P.counts_ws[i];
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, d);
    if (lane == 0) s_excl = (long long)sum;
  }
  process_partition<DT_IN, QUANT, TPP, false, true>(P, part, pt, raw, msk);
  const uint32_t total = partition_scan<C, TPP>(msk, lex, s_wt, s_tile_incl, &s_total);
  const long long excl = s_excl;  // written before the scan's barriers
  const long long off0 = P.hdr->off0;
  if (tid < TPP && part * TPP + tid < P.num_tiles)
    P.prefix[part * TPP + tid + 1] = (uint32_t)(excl + s_tile_incl[tid]);
  if (tid == 0) {
    if (part == 0) P.prefix[0] = 0;
    if (part == P.num_parts - 1) {
      const long long nnz = excl + total;
      if (P.arena_offset) *P.arena_offset = off0 + nnz;
      if (P.vals_offset_out) *P.vals_offset_out = off0;
      if (P.nnz_out) *P.nnz_out = nnz;
    }
  }
  if (P.vals != nullptr)
    write_values<C, PACK>(P, smem_dyn, msk, raw, lex, s_wt, off0 + excl, total,
                          part == P.num_parts - 1 && P.arena_offset == nullptr);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Tiles per partition (a partition is 32 KB of bf16 / fp8 input, 8 KB per
// thread-slot row); MODE 1 / 2 use small partitions.
constexpr int tpp_for(int eb, int mode) {
  return mode == 0 ? (eb == 1 ? 8 : 4) : (eb == 1 ? 2 : 1);
}

template <int DT_IN, bool QUANT, bool PACK, int MODE>
static int launch_t(const CompressParams &P, cudaStream_t st) {
  constexpr int TPP = tpp_for(Elt<DT_IN>::bytes, MODE);
  using C = Cfg<DT_IN, QUANT, TPP>;
  constexpr size_t smem = (MODE == 2) ? 0 : (size_t)TPP * kTileNumel * C::SB + 16;
  static_assert(smem <= 48 * 1024, "stage fits the default dynamic shared memory");
  const unsigned grid = (unsigned)P.num_parts;
  if constexpr (MODE == 0) {
    const size_t nseg = (size_t)((P.num_parts + kSeg - 1) / kSeg);
    if (cudaMemsetAsync(P.seg_ws, 0, nseg * sizeof(unsigned long long), st) != cudaSuccess)
      return BS_ERR_LAUNCH;
    count_kernel<DT_IN, QUANT, PACK, TPP><<<grid, kThreads, 0, st>>>(P);
    if (cudaGetLastError() != cudaSuccess) return BS_ERR_LAUNCH;
    compact_kernel<DT_IN, QUANT, PACK, TPP><<<grid, kThreads, smem, st>>>(P);
  } else {
    compress_kernel<DT_IN, QUANT, PACK, TPP, MODE><<<grid, kThreads, smem, st>>>(P);
  }
  return cudaGetLastError() == cudaSuccess ? BS_OK : BS_ERR_LAUNCH;
}

template <int DT_IN, bool QUANT, int MODE>
static int launch_pack(const CompressParams &P, int pack, cudaStream_t st) {
  return pack ? launch_t<DT_IN, QUANT, true, MODE>(P, st)
              : launch_t<DT_IN, QUANT, false, MODE>(P, st);
}

template <int MODE>
static int dispatch(const CompressParams &P, int dt, bool quant, int pack, cudaStream_t st) {
  if (quant) {
    if (dt == BS_BF16) return launch_pack<BS_BF16, true, MODE>(P, pack, st);
    if (dt == BS_F32) return launch_pack<BS_F32, true, MODE>(P, pack, st);
    return BS_ERR_DTYPE;
  }
  switch (dt) {
    case BS_BF16: return launch_pack<BS_BF16, false, MODE>(P, pack, st);
    case BS_E4M3: return launch_pack<BS_E4M3, false, MODE>(P, pack, st);
    case BS_E5M2: return launch_pack<BS_E5M2, false, MODE>(P, pack, st);
    default: return BS_ERR_DTYPE;
  }
}

static int elt_bytes(int dt) {
  switch (dt) {
    case BS_BF16: return 2;
    case BS_E4M3: case BS_E5M2: return 1;
    case BS_F32: return 4;
    default: return 0;
  }
}

static int fill_common(CompressParams &P, const void *dense, int dt, int64_t M, int64_t N,
                       int64_t ld, int mode) {
  const int eb = elt_bytes(dt);
  if (!eb) return BS_ERR_DTYPE;
  if (M < 0 || N < 0 || ld < N) return BS_ERR_SHAPE;
  if (M > 0 && N > 0 && !dense) return BS_ERR_ARG;
  P.dense = static_cast<const uint8_t *>(dense);
  P.M = M; P.N = N; P.ld = ld;
  P.grid_n = (N + kTileN - 1) / kTileN;
  const int64_t grid_m = (M + kTileM - 1) / kTileM;
  P.num_tiles = grid_m * P.grid_n;
  if (P.num_tiles > (int64_t)1 << 31) return BS_ERR_SHAPE;
  const int tpp = tpp_for(eb, mode);
  P.num_parts = (P.num_tiles + tpp - 1) / tpp;
  // 32-byte vector loads need an aligned base and row stride.
  P.vec_ok = ((reinterpret_cast<uintptr_t>(dense) & 31) == 0) && ((ld * eb) % 32 == 0);
  return BS_OK;
}

}  // namespace bs

using namespace bs;

extern "C" size_t bs_compress_workspace_bytes(int64_t num_tiles) {
  if (num_tiles < 0) num_tiles = 0;
  // Per partition a 4-byte count and per 256 partitions an 8-byte total; a
  // partition holds at least four tiles.
  return sizeof(WsHeader) + 8 * ((size_t)num_tiles / 1024 + 1) + (size_t)num_tiles + 4;
}

extern "C" int bs_compress(const void *dense, int in_dtype, int64_t M, int64_t N, int64_t ld,
                           const float *quant_scale, uint8_t *quant_out, uint8_t *bitmask,
                           uint32_t *prefix, void *vals, int64_t vals_capacity, int pack_sbit,
                           int64_t *arena_offset, int64_t *vals_offset_out, int64_t *nnz_out,
                           void *workspace, size_t workspace_bytes, int32_t *status,
                           void *stream) {
  CompressParams P{};
  int rc = fill_common(P, dense, in_dtype, M, N, ld, 0);
  if (rc) return rc;
  const bool quant = quant_scale != nullptr;
  if (quant && in_dtype != BS_BF16 && in_dtype != BS_F32) return BS_ERR_DTYPE;
  if (!quant && in_dtype == BS_F32) return BS_ERR_DTYPE;
  if (!bitmask || !prefix || !workspace) return BS_ERR_ARG;
  if (pack_sbit != 0 && pack_sbit != 1) return BS_ERR_ARG;
  if (vals_capacity < 0) return BS_ERR_CAPACITY;
  if (pack_sbit && vals && (reinterpret_cast<uintptr_t>(vals) & 3)) return BS_ERR_ALIGN;
  if (pack_sbit && (vals_capacity & 3)) return BS_ERR_ALIGN;
  if (workspace_bytes < bs_compress_workspace_bytes(P.num_parts)) return BS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 15) return BS_ERR_ALIGN;
  P.qscale = quant_scale;
  P.qout = quant_out;
  P.qout_vec = quant_out && ((reinterpret_cast<uintptr_t>(quant_out) & 15) == 0) &&
               (N % 16 == 0);
  P.bitmask = bitmask;
  P.prefix = prefix;
  P.vals = static_cast<uint8_t *>(vals);
  P.cap = vals_capacity;
  P.vals_v16 = (reinterpret_cast<uintptr_t>(vals) & 15) == 0;
  P.arena_offset = arena_offset;
  P.vals_offset_out = vals_offset_out;
  P.nnz_out = nnz_out;
  P.hdr = static_cast<WsHeader *>(workspace);
  P.seg_ws = reinterpret_cast<unsigned long long *>(static_cast<uint8_t *>(workspace) +
                                                     sizeof(WsHeader));
  P.counts_ws = reinterpret_cast<uint32_t *>(P.seg_ws + (P.num_parts + kSeg - 1) / kSeg);
  P.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (P.num_tiles == 0) {
    // Empty tensor: prefix = [0]; arena offset, vals_offset_out, nnz_out untouched.
    if (cudaMemsetAsync(prefix, 0, sizeof(uint32_t), st) != cudaSuccess) return BS_ERR_LAUNCH;
    return BS_OK;
  }
  return dispatch<0>(P, in_dtype, quant, pack_sbit, st);
}

// Reference compact_vals (lib_sparse/src/triton_operators.py:36-115): values
// only, bases from an existing prefix.
extern "C" int bs_compact_vals(const void *dense, int dtype, int64_t M, int64_t N, int64_t ld,
                               const uint32_t *prefix, void *vals, int64_t vals_capacity,
                               int pack_sbit, const int64_t *vals_offset, int32_t *status,
                               void *stream) {
  CompressParams P{};
  int rc = fill_common(P, dense, dtype, M, N, ld, 1);
  if (rc) return rc;
  if (dtype == BS_F32) return BS_ERR_DTYPE;
  if (!prefix) return BS_ERR_ARG;
  if (!vals) return vals_capacity == 0 ? BS_OK : BS_ERR_ARG;  // nothing can be stored
  if (pack_sbit && ((reinterpret_cast<uintptr_t>(vals) & 3) || (vals_capacity & 3)))
    return BS_ERR_ALIGN;
  P.prefix = const_cast<uint32_t *>(prefix);
  P.vals = static_cast<uint8_t *>(vals);
  P.cap = vals_capacity;
  P.vals_v16 = (reinterpret_cast<uintptr_t>(vals) & 15) == 0;
  P.arena_offset = const_cast<int64_t *>(vals_offset);  // read only in MODE 1
  P.status = status;
  if (P.num_tiles == 0) return BS_OK;
  return dispatch<1>(P, dtype, false, pack_sbit, static_cast<cudaStream_t>(stream));
}

extern "C" int bs_tile_pack(const void *dense, int dtype, int64_t M, int64_t N, int64_t ld,
                            int32_t *counts, uint8_t *bitmask, void *stream) {
  CompressParams P{};
  int rc = fill_common(P, dense, dtype, M, N, ld, 2);
  if (rc) return rc;
  if (dtype == BS_F32) return BS_ERR_DTYPE;
  if (P.num_tiles == 0) return BS_OK;
  if (!counts || !bitmask) return BS_ERR_ARG;
  P.counts = counts;
  P.bitmask = bitmask;
  return dispatch<2>(P, dtype, false, 0, static_cast<cudaStream_t>(stream));
}


// ---------------------------------------------------------------------------
// Compress without any allocation: scan scratch in a fixed device array.
//
// For callers that cannot call cudaMalloc (or must not, e.g. code running
// inside an allocator or a framework hook that forbids allocation, and hosts
// that have no device allocator of their own): the fused compressor's scan
// workspace lives in this file-scope array, which every GPU that loads the
// library holds until the process exits.  Inputs and outputs are still the
// caller's.  All calls share the array, so calls that overlap on the GPU
// (different streams, or different host threads on one device) race.
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocMaxTiles = 262144;  // e.g. 16384 x 65536 elements
constexpr size_t kNoAllocScratchBytes =
    sizeof(bs::WsHeader) + (size_t)kNoAllocMaxTiles * sizeof(unsigned long long);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void *g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device.  The symbol's
// host-side name is only a stand-in; the address comes from
// cudaGetSymbolAddress, once per device, with that device current.
int noalloc_scratch(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BS_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return BS_ERR_LAUNCH;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return BS_OK;
}

}  // namespace

extern "C" size_t bs_compress_noalloc_max_tiles(void) { return (size_t)kNoAllocMaxTiles; }

extern "C" int bs_compress_noalloc(const void *dense, int in_dtype, int64_t M, int64_t N,
                                   int64_t ld, const float *quant_scale, uint8_t *quant_out,
                                   uint8_t *bitmask, uint32_t *prefix, void *vals,
                                   int64_t vals_capacity, int pack_sbit, int64_t *arena_offset,
                                   int64_t *vals_offset_out, int64_t *nnz_out, int32_t *status,
                                   void *stream) {
  if (M < 0 || N < 0) return BS_ERR_SHAPE;
  const int64_t tiles = ((M + kTileM - 1) / kTileM) * ((N + kTileN - 1) / kTileN);
  if (tiles > kNoAllocMaxTiles) return BS_ERR_TOO_LARGE;
  void *scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // The compressor leaves its scratch zeroed, but a call that gave up (a
  // bounded wait that expired) may not have; start every call from zero.
  const size_t used = bs_compress_workspace_bytes(tiles);
  if (cudaMemsetAsync(scratch, 0, used, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return BS_ERR_LAUNCH;
  return bs_compress(dense, in_dtype, M, N, ld, quant_scale, quant_out, bitmask, prefix, vals,
                     vals_capacity, pack_sbit, arena_offset, vals_offset_out, nnz_out, scratch,
                     kNoAllocScratchBytes, status, stream);
}
