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
// The fused compress (MODE 0) is one persistent kernel, onepass_kernel
// (described where it is defined), for inputs TMA can read: a 16-byte
// aligned base and a row stride that is a multiple of 16 bytes.  Other
// inputs (and fp32 ones) use two wait-free kernels:
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
// No CTA of these two ever waits for another one; ordering comes from the
// stream.  (BS_COMPRESS_TWO_KERNELS=1 in the environment selects them for
// every input, for comparison.)
//
// Values of the two-kernel path.  Raw storage: staged in shared memory
// already shifted by the destination's misalignment, then written with
// aligned 16-byte stores
// (element stores only for the two edge vectors shared with neighbouring
// partitions).  Packed storage (15/7-bit): re-packed into 32-bit words of the
// continuous bitstream; words shared with a neighbouring partition are merged
// with atomicAnd / atomicOr on disjoint bit masks (order independent).
#include "common.cuh"

#include <cuda_bf16.h>

#include <cuda.h>  // CUtensorMap (types only; the encoder comes through the runtime)

#include <cstdlib>
#include <mutex>

namespace bs {

// Workspace: header {off0, epoch}, uint64 segment totals (zeroed by a memset
// before the count kernel), per-partition counts (uint32 in the two-kernel
// form, cleared after it; epoch-tagged uint64 in the one-pass form).
struct WsHeader {
  long long off0;  // logical index of this tensor's first value
  // one-pass kernel: epoch of the last launch that completed on this
  // workspace (0 in a zeroed workspace); a launch publishes its partition
  // counts tagged with epoch + 1, so the counts of earlier launches read as
  // "not yet published" and the workspace needs no clearing between launches
  unsigned long long epoch;
  unsigned long long pad[14];
};
constexpr int kSeg = 256;  // partitions per segment

struct CompressParams {
  const uint8_t *dense;
  int64_t M, N, ld;
  const float *qscale;
  int qcompiled;  // quantise as the reference's compiled to_fp8 (BS_FP8_COMPILED)
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
  // one-pass bias + ReLU mode: the input is z, the compressed tensor is
  // relu(bf16(z + bias)), which is also written densely to relu_out
  const uint8_t *bias;  // bf16 [N]
  uint8_t *relu_out;    // bf16 [M, N], row stride relu_ld (optional with quant)
  int64_t relu_ld;
  // with quant_out in bias + ReLU mode: quant_out receives e4m3(bf16(h * h)
  // / *qscale2) (the FFN's squared activation) instead of e4m3(h / scale)
  const float *qscale2;
  // per-tile scale mode: scale of each tile (amax_t / 448), written by the
  // one-pass kernel
  float *tile_scales;
  // one-pass kernel: the 3-D tile-column map is valid (N % 64 == 0)
  int box3;
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
      const float r = quant_rcp(qs);
      static_assert(C::VEC % 8 == 0, "groups of eight values");
#pragma unroll
      for (int g = 0; g < C::VEC / 8; ++g) {
        const uint32_t w4[4] = {raw[4 * g], raw[4 * g + 1], raw[4 * g + 2], raw[4 * g + 3]};
        uint32_t o2[2];
        if (P.qcompiled) full_e4m3x8(w4, qs, r, o2);
        else div_e4m3x8(w4, qs, r, o2);
        sv[2 * g] = o2[0];
        sv[2 * g + 1] = o2[1];
      }
    } else {
#pragma unroll
      for (int e = 0; e < C::VEC; ++e) {
        if (P.qcompiled) {
          sv[e >> 2] |= e4m3_compiled(__uint_as_float(raw[e]), qs, quant_rcp(qs)) << (8 * (e & 3));
          continue;
        }
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

// Stage a partition's values (chunk order) in shared memory, starting at
// element `shift` of the stage.
template <typename C>
__device__ __forceinline__ void stage_values(uint8_t *stage, const uint32_t (&msk)[C::S],
                                             const uint32_t (&sv)[C::S][8],
                                             const uint32_t (&lex)[C::S], const uint32_t *s_wt,
                                             int shift) {
  const int warp = threadIdx.x >> 5;
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
}

// Write n staged values to logical value index gbase.  Stage element i holds
// value gbase + i - shift, where shift = gbase % (16 / SB) when PRESHIFTED
// (16-byte destination vectors are then aligned 16-byte stage reads) and 0
// otherwise (each vector is funnel-shifted out of five stage words; the
// stage needs 16 bytes of slack past its values).  `own_tail`: this
// partition owns (and zeroes) the packed stream after its payload up to
// packed_storage_nbytes(nnz) (standalone, last partition).  NT threads
// cooperate; this one is number `tid` of them.
template <typename C, bool PACK, bool PRESHIFTED, int NT = kThreads>
__device__ __forceinline__ void emit_values(const CompressParams &P, const uint8_t *stage,
                                            long long gbase, long long n, bool own_tail,
                                            int tid) {
  if constexpr (!PACK) {
    if (n == 0) return;
    const int shift = PRESHIFTED ? (int)(gbase % C::EPV) : 0;
    const long long cap = P.cap;
    if (tid == 0 && gbase + n > cap) status_or(P.status, BS_STATUS_CAPACITY);
    const long long v0 = gbase / C::EPV;
    const long long v1 = (gbase + n - 1) / C::EPV;
    for (long long v = v0 + tid; v <= v1; v += NT) {
      const long long e0 = v * C::EPV;
      const long long i0 = e0 - gbase + shift;  // stage index of value e0
      if (P.vals_v16 && e0 >= gbase && e0 + C::EPV <= gbase + n && e0 + C::EPV <= cap) {
        uint4 o;
        if constexpr (PRESHIFTED) {
          o = *reinterpret_cast<const uint4 *>(stage + i0 * C::SB);
        } else {
          const uint32_t b = (uint32_t)i0 * C::SB;
          const uint32_t *w = reinterpret_cast<const uint32_t *>(stage) + (b >> 2);
          const uint32_t sh = (b & 3u) * 8u;
          const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
          o.x = __funnelshift_r(w0, w1, sh);
          o.y = __funnelshift_r(w1, w2, sh);
          o.z = __funnelshift_r(w2, w3, sh);
          o.w = __funnelshift_r(w3, w4, sh);
        }
        st_v4(P.vals + e0 * C::SB, o);
      } else {
        for (int e = 0; e < C::EPV; ++e) {
          const long long g = e0 + e;
          if (g >= gbase && g < gbase + n && g < cap) {
            const long long i = i0 + e;
            if constexpr (C::SB == 1) P.vals[g] = stage[i];
            else reinterpret_cast<uint16_t *>(P.vals)[g] =
                reinterpret_cast<const uint16_t *>(stage)[i];
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
    for (long long w = w0 + tid; w <= w1; w += NT) {
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

template <typename C, bool PACK>
__device__ __forceinline__ void write_values(const CompressParams &P, uint8_t *stage,
                                             const uint32_t (&msk)[C::S],
                                             const uint32_t (&sv)[C::S][8],
                                             const uint32_t (&lex)[C::S], const uint32_t *s_wt,
                                             long long gbase, long long n, bool own_tail) {
  stage_values<C>(stage, msk, sv, lex, s_wt, PACK ? 0 : (int)(gbase % C::EPV));
  emit_values<C, PACK, true>(P, stage, gbase, n, own_tail, threadIdx.x);
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
// MODE 0, one pass: a persistent kernel, every CTA resident (a cooperative
// launch).  CTA b owns partitions b, b+G, b+2G, ... (G = grid size; a
// partition is 32 KB of input: 4 bf16 / 8 fp8 tiles).  Per round r
// (partition p = rG + b) the CTA
//   1. has TMA fetch the tiles of partition p + A*G into input stage
//      (r + A) % NS (2-D tiled copies, zero-filled past the tensor's edge),
//   2. prefetches the counts it needs to flush partition q = p - D*G,
//   3. waits for stage r % NS and compacts p IN PLACE: each warp owns RW
//      whole tile rows; in step s lane l takes 8 consecutive elements of row
//      4s + l/8 (one 16-byte shared load), whose 8 mask bits (a bf16x2
//      compare per word) are exactly one bitmask byte; a warp scan of the
//      lanes' counts orders the values.  After a barrier (every row read,
//      warp counts published) each value is stored, predicated, at its
//      partition-wide position -- never past the element it came from --
//      and p's count is published (count + 1, so 0 means "not yet"),
//   4. flushes q: its base is the end of the CTA's own previous partition
//      (q - G) plus the published counts of the G-1 partitions in between.
//      No chain of prefixes runs through the CTAs: a slow CTA delays the
//      others by its counting only, and D rounds of slack absorb that.  The
//      CTA writes q's prefixes and its values (16-byte vectors funnel-shifted
//      out of the stage; only the two edge vectors element by element).
// An earlier single-pass design with a decoupled look-back (a chain of
// inclusive prefixes through the CTAs) reached only ~20% of HBM bandwidth:
// every CTA waited on the slowest of the hundreds of partitions ahead of it.
// ---------------------------------------------------------------------------
// 2-D tiled TMA load of one 64 x 64 tile (no multicast).
__device__ __forceinline__ void tma_load_tile(void *dst, const CUtensorMap *map, int x, int y,
                                              uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
// 3-D tiled TMA load through the tile-column view {64 columns, M rows, N / 64
// tile columns}: a box {64, 64, n} is n horizontally adjacent tiles, landing
// tile-major in shared memory (no multicast).
__device__ __forceinline__ void tma_load_tiles3(void *dst, const CUtensorMap *map, int y, int z,
                                                uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u32(uint32_t *p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// A partition count of the one-pass kernel as published for launch epoch
// `ep`: (ep << 32) | (count + 1).  Returns count + 1, or 0 when the word
// holds no count of this launch yet.
__device__ __forceinline__ uint32_t count_of(unsigned long long w, uint32_t ep) {
  return (uint32_t)(w >> 32) == ep ? (uint32_t)w : 0u;
}

// Shared-memory plan of the one-pass kernel.
template <int DT_IN, bool QUANT, int TPP_, int NW, int D, int A>
struct Onepass {
  static constexpr int EB = Elt<DT_IN>::bytes;
  static constexpr int TPP = TPP_;
  using C = Cfg<DT_IN, QUANT, TPP>;
  static constexpr int SB = C::SB;
  static constexpr int R = TPP * kTileM;          // tile rows per partition
  static constexpr int RW = R / NW;               // rows per warp
  static constexpr int WREG = RW * kTileN * EB;   // bytes of a warp's rows (= its value region)
  static constexpr int IN_BYTES = TPP * kTileNumel * EB;
  // A stage holds a partition from its fetch (A rounds ahead) through its
  // flush (D rounds after it is compacted in place).
  static constexpr int NS = D + 1 + A;
  // per stage: warp counts [NW], tile inclusive counts [TPP], total
  static constexpr int META = NW + TPP + 1;
  // counts a thread reads per flush: the grid is capped at CV * NW * 32 + 1
  static constexpr int CV = 2;
  static constexpr size_t OFF_META = (size_t)NS * IN_BYTES + 32;  // + emit read slack
  static constexpr size_t OFF_BAR = (OFF_META + 4 * NS * META + 7) / 8 * 8;
  static constexpr size_t SMEM = OFF_BAR + 8 * NS;
  static_assert(kTileM % RW == 0 && RW % 4 == 0, "a warp's rows lie in one tile");
  static_assert(SB <= EB, "values fit in place of their inputs");
};

// NT threads write n raw staged values (stage element 0 = value g0): the
// whole 16-byte destination vectors thread-strided, each funnel-shifted out
// of five stage words, then the head and tail elements (the vectors shared
// with the neighbouring ranges) one element per thread.  The stage needs 16 bytes
// of slack past its values; vals must be 16-byte aligned.
template <typename C, int NT>
__device__ __forceinline__ void emit_words(const CompressParams &P, const uint8_t *stage,
                                           long long g0, long long n, int lane) {
  constexpr int EPV = 16 / C::SB;
  if (n <= 0) return;
  const long long cap = P.cap;
  if (g0 + n > cap) {
    if (lane == 0) status_or(P.status, BS_STATUS_CAPACITY);
    n = cap - g0;
    if (n <= 0) return;
  }
  uint8_t *vals = P.vals;
  const int nn = (int)n;                                // < 2^31 (one warp's rows)
  const int head = (int)((EPV - g0 % EPV) % EPV);       // elements before the first vector
  const int nfull = nn > head ? (nn - head) / EPV : 0;  // whole vectors
  const int tail0 = nfull ? head + nfull * EPV : 0;     // first element after them
  const uint32_t *s32 = reinterpret_cast<const uint32_t *>(stage);
  uint4 *dst = reinterpret_cast<uint4 *>(vals + (g0 + head) * C::SB);
  // Vector v starts at stage byte head * SB + 16 v: its word offset within a
  // 16-byte group (o) and byte shift (sh) are the same for every vector, so
  // each lane reads the two aligned 16-byte groups covering its five words
  // (consecutive lanes, consecutive groups: no bank conflicts) and picks the
  // five with a warp-uniform offset.  The reads end at most 16 bytes past
  // the stage's values (slack / the next stage).
  const int rel0 = head * C::SB;
  const int o = (rel0 >> 2) & 3;
  const uint32_t sh = (uint32_t)(rel0 & 3) * 8u;
  for (int v = lane; v < nfull; v += NT) {
    const int j0 = ((rel0 >> 2) & ~3) + 4 * v;  // first word of the aligned group
    const uint4 A = *reinterpret_cast<const uint4 *>(s32 + j0);
    const uint4 B = *reinterpret_cast<const uint4 *>(s32 + j0 + 4);
    uint32_t w0, w1, w2, w3, w4;
    if (o == 0) { w0 = A.x; w1 = A.y; w2 = A.z; w3 = A.w; w4 = B.x; }
    else if (o == 1) { w0 = A.y; w1 = A.z; w2 = A.w; w3 = B.x; w4 = B.y; }
    else if (o == 2) { w0 = A.z; w1 = A.w; w2 = B.x; w3 = B.y; w4 = B.z; }
    else { w0 = A.w; w1 = B.x; w2 = B.y; w3 = B.z; w4 = B.w; }
    dst[v] = make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh),
                        __funnelshift_r(w2, w3, sh), __funnelshift_r(w3, w4, sh));
  }
  // edge elements: [0, head) and [tail0, nn) (all of them when nfull == 0)
  const int nhead = nfull ? head : nn;
  for (int e = lane; e < nhead + (nn - tail0 > 0 && nfull ? nn - tail0 : 0); e += NT) {
    const int i = e < nhead ? e : tail0 + (e - nhead);
    if constexpr (C::SB == 2)
      reinterpret_cast<uint16_t *>(vals)[g0 + i] = reinterpret_cast<const uint16_t *>(stage)[i];
    else
      vals[g0 + i] = stage[i];
  }
}

// Mask of 8 bf16 (4 words): bit i set iff element i > 0 (a bf16x2 compare
// per word: NaN, -0 and +0 give 0).  The compares give 0xFFFF per positive
// halfword; two byte permutes keep one byte per element (element k of the
// first four in byte k of a, of the last four in byte k of b), a mask per
// byte keeps bit k of a's byte k and bit 4 + k of b's, and one multiply by
// 0x01010101 sums the four (disjoint) bytes into the top byte.
__device__ __forceinline__ uint32_t mask_bf16x8(const uint32_t (&w)[4]) {
  const __nv_bfloat162 zero = __float2bfloat162_rn(0.f);
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __hgt2_mask(*reinterpret_cast<const __nv_bfloat162 *>(&w[i]), zero);
  const uint32_t a = __byte_perm(h[0], h[1], 0x6420);
  const uint32_t b = __byte_perm(h[2], h[3], 0x6420);
  const uint32_t y = (a & 0x08040201u) | (b & 0x80402010u);
  return (y * 0x01010101u) >> 24;
}

// Inclusive warp scan: shfl.up's in-range predicate guards each add (no
// branches).
__device__ __forceinline__ uint32_t warp_scan_pred(uint32_t v) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1)
    asm("{\n .reg .u32 t;\n .reg .pred p;\n shfl.sync.up.b32 t|p, %0, %1, 0, 0xffffffff;\n"
        " @p add.u32 %0, %0, t;\n}"
        : "+r"(v)
        : "r"(d));
  return v;
}

// Value placement: when (m & bit) != 0, store v at shared address a and
// advance a by one element; a bit test, a predicated store and a predicated
// add.
__device__ __forceinline__ void place16(uint32_t &a, uint32_t m, uint32_t bit, uint32_t v) {
  asm volatile(
      "{\n .reg .pred p;\n .reg .b32 t;\n and.b32 t, %1, %2;\n setp.ne.u32 p, t, 0;\n"
      " @p st.shared.u16 [%0], %3;\n @p add.u32 %0, %0, 2;\n}"
      : "+r"(a)
      : "r"(m), "r"(bit), "h"((unsigned short)v));
}
__device__ __forceinline__ void place8(uint32_t &a, uint32_t m, uint32_t bit, uint32_t v) {
  asm volatile(
      "{\n .reg .pred p;\n .reg .b32 t;\n and.b32 t, %1, %2;\n setp.ne.u32 p, t, 0;\n"
      " @p st.shared.u8 [%0], %3;\n @p add.u32 %0, %0, 1;\n}"
      : "+r"(a)
      : "r"(m), "r"(bit), "h"((unsigned short)(v & 0xFFu)));
}

template <int DT_IN, bool QUANT, bool PACK, int TPP_, int NW, int D, int A, int MINB,
          bool BIAS = false, bool QC = false, bool TS = false>
__global__ void __launch_bounds__(NW * 32, MINB)
    onepass_kernel(const __grid_constant__ CUtensorMap tmap,
                   const __grid_constant__ CUtensorMap tmap3, const CompressParams P) {
  using O = Onepass<DT_IN, QUANT, TPP_, NW, D, A>;
  using C = typename O::C;
  constexpr int TPP = O::TPP, RW = O::RW, NS = O::NS;
  extern __shared__ __align__(128) uint8_t smem_dyn[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem_dyn + O::OFF_BAR);
  uint32_t *s_meta = reinterpret_cast<uint32_t *>(smem_dyn + O::OFF_META);
  __shared__ uint32_t s_sum[2];  // per round parity: sum of the flush's counts
  __shared__ long long s_off0;
  __shared__ uint32_t s_epoch;
  unsigned long long *cnt64 = reinterpret_cast<unsigned long long *>(P.counts_ws);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long G = gridDim.x, b = blockIdx.x, nparts = P.num_parts;

  // Thread 0 fetches partition `part` into input stage `st`.
  auto fetch = [&](long long part, int st) {
    uint8_t *dst = smem_dyn + (size_t)st * O::IN_BYTES;
    const uint32_t t0 = (uint32_t)(part * TPP), gn = (uint32_t)P.grid_n;  // num_tiles < 2^31
    const int nt = (int)min((long long)TPP, P.num_tiles - (long long)t0);
    mbar_expect_tx(&bars[st], (uint32_t)(nt * kTileNumel * O::EB));
    uint32_t tm = t0 / gn, tn = t0 - tm * gn;
    if (P.box3 && nt == TPP && tn + TPP <= gn) {  // one box: the partition's tiles share a tile row
      tma_load_tiles3(dst, &tmap3, (int)(tm * kTileM), (int)tn, &bars[st]);
      return;
    }
    for (int j = 0; j < nt; ++j) {
      tma_load_tile(dst + j * kTileNumel * O::EB, &tmap, (int)(tn * kTileN), (int)(tm * kTileM),
                    &bars[st]);
      if (++tn == gn) { tn = 0; ++tm; }
    }
  };

  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
    for (int i = 0; i < NS; ++i) mbar_init(&bars[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    long long off = 0;
    if (P.arena_offset) {
      off = *P.arena_offset;
      if (PACK) off = (off + 7) / 8 * 8;  // functions.py:78-81
    }
    s_off0 = off;
    s_sum[0] = 0;
    s_sum[1] = 0;
    uint32_t ep = (uint32_t)*reinterpret_cast<volatile unsigned long long *>(&P.hdr->epoch) + 1u;
    s_epoch = ep ? ep : 1u;
    __threadfence();  // the arena-offset / epoch reads precede every count this CTA publishes
  }
  __syncthreads();
  if (tid == 0)
    for (int i = 0; i < A; ++i)
      if (i * G + b < nparts) fetch(i * G + b, i);

  static_assert(!TS || (QUANT && !BIAS && DT_IN == BS_BF16), "per-tile scales: bf16 input");
  __shared__ uint32_t s_tam[TS ? NW : 1];  // per-tile scale mode: warp amax (bf16 bits)
  const float qs = QUANT && !TS ? *P.qscale : 1.f;
  const float qr = QUANT && !TS ? quant_rcp(qs) : 1.f;
  const float qs2 = (QUANT && BIAS && P.qscale2 != nullptr) ? *P.qscale2 : 1.f;
  const float qr2 = quant_rcp(qs2);
  // the estimate alone quantises exactly at these scales (checked per CTA,
  // while the first partitions are in flight)
  bool qfast = false, qfast2 = false;
  if constexpr (QUANT && !TS) {
    qfast = e4m3_estimate_exact(qs, qr, QC);
    if constexpr (BIAS) qfast2 = P.qscale2 != nullptr && e4m3_estimate_exact(qs2, qr2, QC);
  }
  const uint32_t epoch = s_epoch;
  long long known_end = 0, known = -1;  // end (count) through this CTA's last flushed partition
  for (long long r = 0;; ++r) {
    const long long p = r * G + b;
    const long long q = p - (long long)D * G;
    if (q >= nparts) break;
    if (tid == 0) {
      const long long pf = p + (long long)A * G;
      // the stage's last reads were ordered by the round's closing barrier
      if (pf < nparts) fetch(pf, (int)((r + A) % NS));
    }
    // 2. counts of the partitions between this CTA's last flushed one and q
    //    (G - 1 of them; a thread reads at most kCv).  The raw words are
    //    only decoded at the flush: a use here would hold every warp for an
    //    L2 round trip (~1.7k cycles per round, measured) before compaction.
    constexpr int kCv = O::CV;
    const unsigned long long kOne = ((unsigned long long)epoch << 32) | 1u;  // "count 0"
    unsigned long long cw[kCv];
#pragma unroll
    for (int i = 0; i < kCv; ++i) {
      const long long ci = known + 1 + tid + (long long)i * NW * 32;
      cw[i] = (q >= 0 && ci < q) ? ld_relaxed_u64(cnt64 + ci) : kOne;
    }
    // 3. compact partition p in place
    if (p < nparts) {
      const int st = (int)(r % NS);
      const int rho0 = warp * RW;  // first partition row of this warp
      const int j = rho0 / kTileM;  // its tile
      const long long tile = p * TPP + j;
      const int sub = lane >> 3, c8 = lane & 7;
      const bool valid = tile < P.num_tiles;  // warp-uniform
      // bias + ReLU mode: this lane's 8 columns are the same in every step;
      // the bias is loaded before the stage wait (its latency overlaps it)
      uint32_t bw[4] = {0, 0, 0, 0};
      int64_t brow0 = 0, bcol = 0;
      if constexpr (BIAS) {
        if (valid) {
          const int64_t tm = tile / P.grid_n, tn = tile - tm * P.grid_n;
          brow0 = tm * kTileM + (rho0 - j * kTileM) + sub;
          bcol = tn * kTileN + 8 * c8;
          if (bcol + 8 <= P.N) {
            const uint4 b4 = *reinterpret_cast<const uint4 *>(P.bias + bcol * 2);
            bw[0] = b4.x; bw[1] = b4.y; bw[2] = b4.z; bw[3] = b4.w;
          } else {
            for (int i = 0; i < 8; ++i)
              if (bcol + i < P.N)
                bw[i >> 1] |= (uint32_t)reinterpret_cast<const uint16_t *>(P.bias)[bcol + i]
                              << (16 * (i & 1));
          }
        }
      }
      {
        bool ok = false;
        for (uint32_t n = 0; n < kMaxPolls && !(ok = mbar_try_wait(&bars[st], (uint32_t)((r / NS) & 1))); ++n) {
        }
        if (!ok && tid == 0) status_or(P.status, BS_STATUS_TIMEOUT);
      }
      uint8_t *stage = smem_dyn + (size_t)st * O::IN_BYTES;
      uint32_t *meta = s_meta + st * O::META;
      // lane: 8 consecutive elements (16 B of bf16 / 8 B of fp8) of row
      // rho0 + 4s + lane / 8 in step s; its 8 mask bits are exactly one
      // bitmask byte.  All of a warp's rows are read before the barrier
      // below, after which values are written in place at their
      // partition-wide positions (never past the element they came from).
      constexpr int S = RW / 4;
      constexpr int VW = O::EB == 2 ? 4 : 2;  // input words per lane and step
      uint32_t v[S][VW], m[S], ex[S];
      uint32_t wtot = 0;
      if (valid) {
        uint8_t *bm = P.bitmask + (p * TPP * kTileM + rho0 + sub) * 8 + c8;
#pragma unroll
        for (int s4 = 0; s4 < S; ++s4) {
          const uint8_t *src = stage + ((rho0 + 4 * s4 + sub) * kTileN + 8 * c8) * O::EB;
          if constexpr (VW == 4) {
            const uint4 w = *reinterpret_cast<const uint4 *>(src);
            v[s4][0] = w.x; v[s4][1] = w.y; v[s4][2] = w.z; v[s4][3] = w.w;
          } else {
            const uint2 w = *reinterpret_cast<const uint2 *>(src);
            v[s4][0] = w.x; v[s4][1] = w.y;
          }
        }
        // per-tile scale mode: amax of the tile (NaN ignored) from its warps'
        // rows, then scale = amax / 448 and the code is e4m3(x * (448 / amax))
        // (a zero tile: scale 1, every code 0)
        float tinv = 0.f;
        if constexpr (TS) {
          uint32_t am = 0;
#pragma unroll
          for (int s4 = 0; s4 < S; ++s4)
#pragma unroll
            for (int i = 0; i < VW; ++i) {
              uint32_t lo = v[s4][i] & 0x7FFFu, hi = (v[s4][i] >> 16) & 0x7FFFu;
              lo = lo > 0x7F80u ? 0u : lo;
              hi = hi > 0x7F80u ? 0u : hi;
              am = max(am, max(lo, hi));
            }
          am = __reduce_max_sync(0xFFFFFFFFu, am);
          constexpr int WPT = kTileM / RW;  // warps per tile, all valid or all not
          if (lane == 0) s_tam[warp] = am;
          asm volatile("bar.sync %0, %1;" ::"r"(1 + j), "r"(WPT * 32) : "memory");
#pragma unroll
          for (int k = 0; k < WPT; ++k) am = max(am, s_tam[j * WPT + k]);
          const float a = __uint_as_float(am << 16);
          tinv = a > 0.f ? __fdiv_rn(448.f, a) : 0.f;
          if (lane == 0 && rho0 == j * kTileM) P.tile_scales[tile] = a > 0.f ? __fdiv_rn(a, 448.f) : 1.f;
        }
#pragma unroll
        for (int s4 = 0; s4 < S; ++s4) {
          if constexpr (BIAS) {
            // y = relu(bf16(z + bias)): fp32 add rounded once to bf16 (torch's
            // bf16 add), then strictly negative values -> +0 (-0 and NaN kept)
            const int64_t grow = brow0 + 4 * s4;
            // rows past M (TMA zero fill) stay 0: the bias must not reach them
            const uint32_t live = grow < P.M ? 0xFFFFFFFFu : 0u;
#pragma unroll
            for (int i = 0; i < 4; ++i) v[s4][i] = relu_bf16x2(bf16x2_add(v[s4][i], bw[i])) & live;
            if (P.relu_out != nullptr && grow < P.M) {
              uint8_t *dst = P.relu_out + (grow * P.relu_ld + bcol) * 2;
              if (bcol + 8 <= P.N) {
                *reinterpret_cast<uint4 *>(dst) = make_uint4(v[s4][0], v[s4][1], v[s4][2], v[s4][3]);
              } else {
                for (int i = 0; i < 8; ++i)
                  if (bcol + i < P.N)
                    reinterpret_cast<uint16_t *>(dst)[i] = (uint16_t)(v[s4][i >> 1] >> (16 * (i & 1)));
              }
            }
          }
          if constexpr (QUANT) {
            uint32_t qw[2] = {0, 0}, side[2];
            {
              const uint32_t h4[4] = {v[s4][0], v[s4][1], v[s4][2], v[s4][3]};
              if constexpr (TS) {
                est_e4m3x8<true>(h4, tinv, qw);  // e4m3(x * inv_t), round to nearest even
              } else if (qfast) {
                est_e4m3x8<QC>(h4, qr, qw);
              } else {
                const uint2 c = quant8_checked(h4[0], h4[1], h4[2], h4[3], qs, qr, QC);
                qw[0] = c.x;
                qw[1] = c.y;
              }
            }
            side[0] = qw[0];
            side[1] = qw[1];
            if constexpr (BIAS) {
              if (P.qscale2 != nullptr) {
                // side output: e4m3(bf16(h * h) / scale2) (h.square_() then to_fp8)
                uint32_t sq[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) sq[i] = bf16x2_mul(v[s4][i], v[s4][i]);  // h.square_()
                if (qfast2) {
                  est_e4m3x8<QC>(sq, qr2, side);
                } else {
                  const uint2 c = quant8_checked(sq[0], sq[1], sq[2], sq[3], qs2, qr2, QC);
                  side[0] = c.x;
                  side[1] = c.y;
                }
              }
            }
            v[s4][0] = qw[0]; v[s4][1] = qw[1];
            if (P.qout) {
              const long long tm = tile / P.grid_n, tn = tile - tm * P.grid_n;
              const long long gcol = tn * kTileN + 8 * c8;
              const long long grow = tm * kTileM + (rho0 + 4 * s4 + sub - j * kTileM);
              if (grow < P.M) {
                uint8_t *qo = P.qout + grow * P.N + gcol;
                if (P.qout_vec && gcol + 8 <= P.N) {
                  *reinterpret_cast<uint2 *>(qo) = make_uint2(side[0], side[1]);
                } else {
#pragma unroll
                  for (int i = 0; i < 8; ++i)
                    if (gcol + i < P.N) qo[i] = (uint8_t)(side[i >> 2] >> (8 * (i & 3)));
                }
              }
            }
          }
          uint32_t mm;
          if constexpr (C::SB == 2) {
            mm = mask_bf16x8(v[s4]);
          } else {
            const uint32_t w2[2] = {v[s4][0], v[s4][1]};
            mm = mask_of_words<C::SDT, 2>(w2);
          }
          m[s4] = mm;
          bm[s4 * 32] = (uint8_t)mm;
        }
        // Lane counts of three steps share one scan: 10-bit fields (a
        // step's inclusive count is at most 256, so fields never carry).
#pragma unroll
        for (int g = 0; g < S; g += 3) {
          uint32_t packed = 0;
#pragma unroll
          for (int k = 0; k < 3 && g + k < S; ++k) packed |= (uint32_t)__popc(m[g + k]) << (10 * k);
          const uint32_t incl = warp_scan_pred(packed);
          const uint32_t tot = __shfl_sync(0xFFFFFFFFu, incl, 31);
#pragma unroll
          for (int k = 0; k < 3 && g + k < S; ++k) {
            ex[g + k] = wtot + ((incl - packed) >> (10 * k) & 0x3FFu);
            wtot += (tot >> (10 * k)) & 0x3FFu;
          }
        }
      }
      if (lane == 0) meta[warp] = wtot;
      __syncthreads();  // all rows read; warp counts published
      if (tid == 0) {
        uint32_t acc = 0;
#pragma unroll
        for (int t = 0; t < TPP; ++t) {
#pragma unroll
          for (int w = t * (kTileM / RW); w < (t + 1) * (kTileM / RW); ++w) acc += meta[w];
          meta[NW + t] = acc;  // inclusive count after tile t
        }
        meta[NW + TPP] = acc;
        st_relaxed_u64(cnt64 + p, ((unsigned long long)epoch << 32) | (acc + 1));
      }
      if (valid && P.vals != nullptr) {
        const uint32_t t = lane < warp ? meta[lane] : 0u;
        const uint32_t wex = __reduce_add_sync(0xFFFFFFFFu, t);
        const uint32_t base_addr = smem_addr(stage);
        // The placement stores are volatile asm (kept in program order), so
        // the S steps' independent address chains are interleaved here:
        // element i of every step, then element i + 1 -- each chain's
        // dependent add is S stores behind its predecessor.
        uint32_t a[S];
#pragma unroll
        for (int s4 = 0; s4 < S; ++s4) a[s4] = base_addr + (wex + ex[s4]) * C::SB;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
#pragma unroll
          for (int s4 = 0; s4 < S; ++s4) {
            if constexpr (C::SB == 2) place16(a[s4], m[s4], 1u << i, v[s4][i >> 1] >> (16 * (i & 1)));
            else place8(a[s4], m[s4], 1u << i, v[s4][i >> 2] >> (8 * (i & 3)));
          }
        }
      }
    }

    // 4. flush partition q
    if (q >= 0) {
      const int slot = (int)((r - D) % NS);
      const uint32_t *meta = s_meta + slot * O::META;  // written before an earlier barrier
      bool late = false;
      uint32_t sum = 0;
      uint32_t cv[kCv];
#pragma unroll
      for (int i = 0; i < kCv; ++i) cv[i] = count_of(cw[i], epoch);
#pragma unroll
      for (int i = 0; i < kCv; ++i) {
        const long long ci = known + 1 + tid + (long long)i * NW * 32;
        for (uint32_t n = 0; cv[i] == 0; ++n) {  // published yet?  (0 only for ci < q)
          if (n >= kMaxPolls) { late = true; cv[i] = 1; break; }
          __nanosleep(64);
          cv[i] = count_of(ld_relaxed_u64(cnt64 + ci), epoch);
        }
        sum += cv[i] - 1;
      }
      if (late) status_or(P.status, BS_STATUS_TIMEOUT);
      sum = __reduce_add_sync(0xFFFFFFFFu, sum);
      if (lane == 0 && sum) atomicAdd(&s_sum[r & 1], sum);
      __syncthreads();
      long long base = known_end + s_sum[r & 1];
      const uint32_t total = meta[NW + TPP];
      const long long off0 = s_off0;
      if (tid < TPP && q * TPP + tid < P.num_tiles)
        P.prefix[q * TPP + tid + 1] = (uint32_t)(base + meta[NW + tid]);
      if (tid == 0) {
        if (q == 0) P.prefix[0] = 0;
        if (q == nparts - 1) {
          __threadfence();
          const long long nnz = base + total;
          if (P.arena_offset) *P.arena_offset = off0 + nnz;
          if (P.vals_offset_out) *P.vals_offset_out = off0;
          if (P.nnz_out) *P.nnz_out = nnz;
          // every CTA has read the epoch: this flush needed a count from each
          *reinterpret_cast<volatile unsigned long long *>(&P.hdr->epoch) = epoch;
        }
      }
      if (P.vals != nullptr) {
        const uint8_t *vs = smem_dyn + (size_t)slot * O::IN_BYTES;
        if constexpr (PACK)
          emit_values<C, true, false, NW * 32>(P, vs, off0 + base, total,
                                               q == nparts - 1 && P.arena_offset == nullptr, tid);
        else
          emit_words<C, NW * 32>(P, vs, off0 + base, total, tid);
      }
      known_end = base + total;
      known = q;
    }
    if (tid == 0) s_sum[(r + 1) & 1] = 0;  // next round's accumulator (read this round: the other)
    fence_proxy_async_smem();  // this round's stage accesses precede the next TMA writes
    __syncthreads();  // stage (r-D) % NS and s_sum are free again
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Tiles per partition (a partition is 32 KB of bf16 / fp8 input, 8 KB per
// thread-slot row); MODE 1 / 2 use small partitions.
constexpr int tpp_for(int eb, int mode) {
  return mode == 0 ? (eb == 1 ? 8 : 4) : (eb == 1 ? 2 : 1);
}

// Resident CTAs of `kernel` on this device: cached per kernel and device
// (the first query also raises the kernel's dynamic shared-memory limit).
static int resident_ctas(const void *kernel, size_t smem, int threads) {
  constexpr int kMaxDev = 64, kMaxKernels = 64;
  static std::mutex mu;
  static const void *keys[kMaxKernels] = {};
  static int cache[kMaxKernels][kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 0;
  std::lock_guard<std::mutex> lock(mu);
  int k = 0;
  while (k < kMaxKernels && keys[k] && keys[k] != kernel) ++k;
  if (k == kMaxKernels) return 0;
  keys[k] = kernel;
  if (!cache[k][dev]) {
    int sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) !=
        cudaSuccess)
      return 0;
    cache[k][dev] = sms * per_sm;
  }
  return cache[k][dev];
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver, through the runtime (no -lcuda).
static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

constexpr int kNotApplicable = -1;


// The one-pass kernel, or kNotApplicable when the input cannot be read by
// TMA (base not 16-byte aligned, row stride not a multiple of 16 bytes,
// sizes past the tensor map's limits) or raw values are not 16-byte aligned.
// TPP2: tiles per partition for 2-byte inputs (1-byte inputs take twice as
// many while a warp's rows stay within one tile); NW warps per CTA; flush
// lag D; prefetch depth A.
template <int DT_IN, int TPP2, int NW>
constexpr int onepass_tpp() {
  return Elt<DT_IN>::bytes == 1 && 2 * TPP2 * kTileM / NW <= kTileM ? 2 * TPP2 : TPP2;
}

template <int DT_IN, bool QUANT, bool PACK, int TPP2, int NW, int D, int A, int MINB = 2,
          bool BIAS = false, bool TS = false>
static int launch_onepass(const CompressParams &P, cudaStream_t st) {
  constexpr int TPP = onepass_tpp<DT_IN, TPP2, NW>();
  using O = Onepass<DT_IN, QUANT, TPP, NW, D, A>;
  if (getenv("BS_COMPRESS_TWO_KERNELS")) return kNotApplicable;
  const uint64_t row_bytes = (uint64_t)P.ld * O::EB;
  if ((reinterpret_cast<uintptr_t>(P.dense) & 15) || (row_bytes & 15) ||
      (!PACK && (reinterpret_cast<uintptr_t>(P.vals) & 15)) || P.M >= ((int64_t)1 << 31) ||
      P.N >= ((int64_t)1 << 31) || row_bytes >= ((uint64_t)1 << 40))
    return kNotApplicable;
  EncodeTiledFn encode = encode_tiled();
  if (!encode) return kNotApplicable;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)P.N, (cuuint64_t)P.M};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {kTileN, kTileM};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType ty =
      O::EB == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  if (encode(&map, ty, 2, const_cast<uint8_t *>(P.dense), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, promo,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return kNotApplicable;
  // The tile-column view {64 columns, M rows, N / 64 tile columns} with
  // strides (row, tile column) = (row_bytes, 64 elements), for whole tile
  // columns only: a partition whose tiles share a tile row is then one TMA
  // box instead of TPP (measured 2-4% faster at 50-99% sparsity on 8192 x
  // 14336 bf16; the four-tile loads remain for partitions that wrap a row).
  CUtensorMap map3 = map;
  int box3 = 0;
  if (P.N % kTileN == 0) {
    const cuuint64_t dims3[3] = {(cuuint64_t)kTileN, (cuuint64_t)P.M, (cuuint64_t)(P.N / kTileN)};
    const cuuint64_t strides3[2] = {(cuuint64_t)row_bytes, (cuuint64_t)(kTileN * O::EB)};
    const cuuint32_t box3d[3] = {kTileN, kTileM, (cuuint32_t)O::TPP};
    const cuuint32_t estr3[3] = {1, 1, 1};
    box3 = encode(&map3, ty, 3, const_cast<uint8_t *>(P.dense), dims3, strides3, box3d, estr3,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, promo,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    if (!box3) map3 = map;
  }
  auto kernel = onepass_kernel<DT_IN, QUANT, PACK, TPP, NW, D, A, MINB, BIAS, false, TS>;
  if constexpr (QUANT && !TS) {  // the compiled to_fp8's quantiser: its own instantiation
    if (P.qcompiled) kernel = onepass_kernel<DT_IN, QUANT, PACK, TPP, NW, D, A, MINB, BIAS, true>;
  }
  int resident = resident_ctas(reinterpret_cast<const void *>(kernel), O::SMEM, NW * 32);
  if (resident <= 0) return BS_ERR_LAUNCH;
  // a flush reads the counts of G - 1 partitions, at most CV per thread
  if (resident > O::CV * NW * 32 + 1) resident = O::CV * NW * 32 + 1;
  CompressParams Q = P;
  Q.num_parts = (P.num_tiles + O::TPP - 1) / O::TPP;
  Q.box3 = box3;
  // counts are published as 64-bit epoch-tagged words (no clearing needed);
  // a partition holds at least four tiles, so they fit in the 2 bytes per
  // tile that bs_compress_workspace_bytes provides
  static_assert(O::TPP >= 4, "8-byte counts need at least four tiles per partition");
  // Every CTA waits on counts that others publish: all must be resident,
  // which a cooperative launch guarantees (or refuses).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(Q.num_parts < resident ? Q.num_parts : resident));
  cfg.blockDim = dim3(NW * 32);
  cfg.dynamicSmemBytes = O::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, map, map3, Q) != cudaSuccess) return BS_ERR_LAUNCH;
  return BS_OK;
}

template <int DT_IN, bool QUANT, bool PACK, int MODE>
static int launch_t(const CompressParams &P, cudaStream_t st) {
  constexpr int TPP = tpp_for(Elt<DT_IN>::bytes, MODE);
  using C = Cfg<DT_IN, QUANT, TPP>;
  constexpr size_t smem = (MODE == 2) ? 0 : (size_t)TPP * kTileNumel * C::SB + 16;
  static_assert(smem <= 48 * 1024, "stage fits the default dynamic shared memory");
  const unsigned grid = (unsigned)P.num_parts;
  if constexpr (MODE == 0) {
    if constexpr (DT_IN != BS_F32) {
      const int rc = launch_onepass<DT_IN, QUANT, PACK, 4, 8, 1, 1>(P, st);
      if (rc != kNotApplicable) return rc;
    }
    const size_t nseg = (size_t)((P.num_parts + kSeg - 1) / kSeg);
    if (cudaMemsetAsync(P.seg_ws, 0, nseg * sizeof(unsigned long long), st) != cudaSuccess)
      return BS_ERR_LAUNCH;
    count_kernel<DT_IN, QUANT, PACK, TPP><<<grid, kThreads, 0, st>>>(P);
    if (cudaGetLastError() != cudaSuccess) return BS_ERR_LAUNCH;
    compact_kernel<DT_IN, QUANT, PACK, TPP><<<grid, kThreads, smem, st>>>(P);
    if (cudaGetLastError() != cudaSuccess) return BS_ERR_LAUNCH;
    // leave the counts zero: the one-pass kernel reads these words as
    // epoch-tagged 64-bit counts, and plain counts must not look like one
    if (cudaMemsetAsync(P.counts_ws, 0, (size_t)P.num_parts * sizeof(uint32_t), st) !=
        cudaSuccess)
      return BS_ERR_LAUNCH;
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
  // bound the factors before multiplying (M, N near 2^62 would wrap)
  if (P.grid_n > 0 && grid_m > ((int64_t)1 << 31) / P.grid_n) return BS_ERR_SHAPE;
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
  // Per 256 partitions an 8-byte total and per partition a 4-byte count; a
  // partition holds at least two tiles.
  return sizeof(WsHeader) + 8 * ((size_t)num_tiles / 512 + 1) + 2 * (size_t)num_tiles + 4;
}

namespace bs {
// Argument checks and parameter block shared by bs_compress and
// bs_compress_bias_relu.
static int setup_compress(CompressParams &P, const void *dense, int in_dtype, int64_t M,
                          int64_t N, int64_t ld, const float *quant_scale, uint8_t *quant_out,
                          uint8_t *bitmask, uint32_t *prefix, void *vals,
                          int64_t vals_capacity, int pack_sbit, int64_t *arena_offset,
                          int64_t *vals_offset_out, int64_t *nnz_out, void *workspace,
                          size_t workspace_bytes, int32_t *status) {
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
  if (workspace_bytes < bs_compress_workspace_bytes(P.num_tiles)) return BS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 15) return BS_ERR_ALIGN;
  P.qscale = quant_scale;
  P.qout = quant_out;
  P.qcompiled = 0;
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
  return BS_OK;
}
}  // namespace bs

extern "C" int bs_compress(const void *dense, int in_dtype, int64_t M, int64_t N, int64_t ld,
                           const float *quant_scale, uint8_t *quant_out, uint8_t *bitmask,
                           uint32_t *prefix, void *vals, int64_t vals_capacity, int pack_sbit,
                           int64_t *arena_offset, int64_t *vals_offset_out, int64_t *nnz_out,
                           void *workspace, size_t workspace_bytes, int32_t *status,
                           void *stream) {
  const int qcompiled = (in_dtype & BS_FP8_COMPILED) != 0;
  in_dtype &= ~BS_FP8_COMPILED;
  CompressParams P{};
  const int rc = setup_compress(P, dense, in_dtype, M, N, ld, quant_scale, quant_out, bitmask,
                                prefix, vals, vals_capacity, pack_sbit, arena_offset,
                                vals_offset_out, nnz_out, workspace, workspace_bytes, status);
  if (rc) return rc;
  P.qcompiled = qcompiled;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (P.num_tiles == 0) {
    // Empty tensor: prefix = [0]; arena offset, vals_offset_out, nnz_out untouched.
    if (cudaMemsetAsync(prefix, 0, sizeof(uint32_t), st) != cudaSuccess) return BS_ERR_LAUNCH;
    return BS_OK;
  }
  return dispatch<0>(P, in_dtype, quant_scale != nullptr, pack_sbit, st);
}

extern "C" int bs_compress_bias_relu(const void *z, int64_t M, int64_t N, int64_t ld,
                                     const void *bias, void *relu_out, int64_t relu_ld,
                                     uint8_t *bitmask, uint32_t *prefix, void *vals,
                                     int64_t vals_capacity, int pack_sbit,
                                     int64_t *arena_offset, int64_t *vals_offset_out,
                                     int64_t *nnz_out, void *workspace, size_t workspace_bytes,
                                     int32_t *status, void *stream) {
  CompressParams P{};
  int rc = setup_compress(P, z, BS_BF16, M, N, ld, nullptr, nullptr, bitmask, prefix, vals,
                          vals_capacity, pack_sbit, arena_offset, vals_offset_out, nnz_out,
                          workspace, workspace_bytes, status);
  if (rc) return rc;
  if (!bias || !relu_out) return BS_ERR_ARG;
  if (relu_ld < N) return BS_ERR_SHAPE;
  // 16-byte bias loads and dense stores
  if ((reinterpret_cast<uintptr_t>(bias) & 15) || (reinterpret_cast<uintptr_t>(relu_out) & 15) ||
      ((relu_ld * 2) & 15))
    return BS_ERR_ALIGN;
  P.bias = static_cast<const uint8_t *>(bias);
  P.relu_out = static_cast<uint8_t *>(relu_out);
  P.relu_ld = relu_ld;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (P.num_tiles == 0) {
    if (cudaMemsetAsync(prefix, 0, sizeof(uint32_t), st) != cudaSuccess) return BS_ERR_LAUNCH;
    return BS_OK;
  }
  // one pass only; BS_ERR_ALIGN when TMA cannot read z (the caller then
  // applies bias and ReLU itself and calls bs_compress)
  rc = pack_sbit ? launch_onepass<BS_BF16, false, true, 4, 8, 1, 1, 2, true>(P, st)
                 : launch_onepass<BS_BF16, false, false, 4, 8, 1, 1, 2, true>(P, st);
  return rc == kNotApplicable ? BS_ERR_ALIGN : rc;
}

extern "C" int bs_compress_fp8_tile_scaled(const void *dense, int64_t M, int64_t N, int64_t ld,
                                           float *tile_scales, uint8_t *bitmask, uint32_t *prefix,
                                           void *vals, int64_t vals_capacity, int pack_sbit,
                                           int64_t *arena_offset, int64_t *vals_offset_out,
                                           int64_t *nnz_out, void *workspace,
                                           size_t workspace_bytes, int32_t *status,
                                           void *stream) {
  if (!tile_scales) return BS_ERR_ARG;
  CompressParams P{};
  // (tile_scales stands in for the quantiser's scale: e4m3 storage; the
  // kernel never reads it as a scale)
  const int rc = setup_compress(P, dense, BS_BF16, M, N, ld, tile_scales, nullptr, bitmask,
                                prefix, vals, vals_capacity, pack_sbit, arena_offset,
                                vals_offset_out, nnz_out, workspace, workspace_bytes, status);
  if (rc) return rc;
  P.tile_scales = tile_scales;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (P.num_tiles == 0) {
    if (cudaMemsetAsync(prefix, 0, sizeof(uint32_t), st) != cudaSuccess) return BS_ERR_LAUNCH;
    return BS_OK;
  }
  // one pass only; BS_ERR_ALIGN when TMA cannot read the input
  const int r = pack_sbit ? launch_onepass<BS_BF16, true, true, 4, 8, 1, 1, 2, false, true>(P, st)
                          : launch_onepass<BS_BF16, true, false, 4, 8, 1, 1, 2, false, true>(P, st);
  return r == kNotApplicable ? BS_ERR_ALIGN : r;
}

extern "C" int bs_compress_bias_relu_fp8(const void *z, int64_t M, int64_t N, int64_t ld,
                                         const void *bias, const float *scale_h,
                                         const float *scale_side, uint8_t *side_out,
                                         uint8_t *bitmask, uint32_t *prefix, void *vals,
                                         int64_t vals_capacity, int pack_sbit,
                                         int64_t *arena_offset, int64_t *vals_offset_out,
                                         int64_t *nnz_out, void *workspace,
                                         size_t workspace_bytes, int fp8_flags,
                                         int32_t *status, void *stream) {
  CompressParams P{};
  if (!scale_h) return BS_ERR_ARG;
  int rc = setup_compress(P, z, BS_BF16, M, N, ld, scale_h, side_out, bitmask, prefix, vals,
                          vals_capacity, pack_sbit, arena_offset, vals_offset_out, nnz_out,
                          workspace, workspace_bytes, status);
  if (rc) return rc;
  if (!bias) return BS_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(bias) & 15) return BS_ERR_ALIGN;
  P.bias = static_cast<const uint8_t *>(bias);
  P.qscale2 = scale_side;
  P.qcompiled = (fp8_flags & BS_FP8_COMPILED) != 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (P.num_tiles == 0) {
    if (cudaMemsetAsync(prefix, 0, sizeof(uint32_t), st) != cudaSuccess) return BS_ERR_LAUNCH;
    return BS_OK;
  }
  rc = pack_sbit ? launch_onepass<BS_BF16, true, true, 4, 8, 1, 1, 2, true>(P, st)
                 : launch_onepass<BS_BF16, true, false, 4, 8, 1, 1, 2, true>(P, st);
  return rc == kNotApplicable ? BS_ERR_ALIGN : rc;
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
// cudaGetSymbolAddress, once per device, with that device current.  The
// cached address is not refreshed after cudaDeviceReset: a process that
// resets a device must not call bs_compress_noalloc on it again.
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
  const int qcompiled = (in_dtype & BS_FP8_COMPILED) != 0;
  in_dtype &= ~BS_FP8_COMPILED;
  if (M < 0 || N < 0) return BS_ERR_SHAPE;
  const int64_t gm = (M + kTileM - 1) / kTileM, gn = (N + kTileN - 1) / kTileN;
  // bound the factors one at a time: their product could wrap
  if (gn > 0 && gm > kNoAllocMaxTiles / gn) return BS_ERR_TOO_LARGE;
  void *scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // Every host-side check runs before anything is queued: a call that is
  // refused leaves the shared array alone.
  CompressParams P{};
  rc = setup_compress(P, dense, in_dtype, M, N, ld, quant_scale, quant_out, bitmask, prefix, vals,
                      vals_capacity, pack_sbit, arena_offset, vals_offset_out, nnz_out, scratch,
                      kNoAllocScratchBytes, status);
  if (rc) return rc;
  P.qcompiled = qcompiled;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (P.num_tiles == 0) {
    if (cudaMemsetAsync(prefix, 0, sizeof(uint32_t), st) != cudaSuccess) return BS_ERR_LAUNCH;
    return BS_OK;
  }
  // The compressor leaves its scratch zeroed, but a call that gave up (a
  // bounded wait that expired) may not have; start every call from zero.
  if (cudaMemsetAsync(scratch, 0, bs_compress_workspace_bytes(P.num_tiles), st) != cudaSuccess)
    return BS_ERR_LAUNCH;
  return dispatch<0>(P, in_dtype, quant_scale != nullptr, pack_sbit, st);
}
