// K1 -- fused single-pass compress: dense -> bitmask, prefix, compacted values.
//
// Reference behaviour replaced (Maxzhu123/bitsparse):
//   _tile_pack_kernel     lib_sparse/src/triton_kernels.py:63-97
//   torch.cumsum prefix   lib_sparse/src/functions.py:33-40
//   _compact_vals_kernel  lib_sparse/src/triton_kernels.py:105-146
//   _pack_kernel          lib_sparse/src/bitpacking.py:58-117
//   arena offset update   lib_sparse/src/functions.py:73-92
// The reference reads the dense tensor twice (tile_pack, then compact) with a
// library scan in between; this kernel reads it once.
//
// Work decomposition.  A CTA of 256 threads owns a "partition" of TPP
// consecutive tiles (tile id order = output order), handed out by an atomic
// ticket: partition p is only processed by a CTA that started after the
// CTAs of partitions < p, so the look-back below only waits on CTAs that are
// already running.  Each thread owns 32-byte chunks (16 bf16 / 32 fp8 / 8
// fp32 elements of one tile row), read with one 256-bit load; a warp covers
// whole tile rows, so every DRAM sector is used in full.  A chunk's mask bits
// are exactly its 2 / 4 / 1 bitmask bytes in the reference's LSB-first,
// row-major-in-tile order; they are computed with SWAR integer arithmetic
// on the raw bits (x > 0 <=> 0 < bits <= +inf / max-finite).
//
// Offsets.  A block-wide exclusive scan of chunk popcounts in (tile, chunk)
// order gives each chunk's offset inside the partition.  The partition's
// total is published as a packed 64-bit status word {state, value} and the
// WHOLE CTA looks back over 256 predecessors per round (single-pass scan
// with decoupled look-back).  A look-back round costs about one L2 round
// trip; the rate at which partitions can retire is bounded by window / round
// time, and on B200 a one-warp window of 32 would cap this kernel well below
// HBM bandwidth -- 256 keeps the scan off the critical path.  Waits are
// bounded (kMaxPolls): on expiry the CTA records BS_STATUS_TIMEOUT and goes
// on, so no CTA spins forever.
//
// Values.  Raw storage: staged in shared memory already shifted by the
// destination's misalignment, then written with aligned 16-byte stores
// (element stores only for the two edge vectors shared with neighbouring
// partitions).  Packed storage (15/7-bit): the staged values are re-packed
// into 32-bit words of the continuous bitstream; words shared with a
// neighbouring partition are merged with atomicAnd / atomicOr on disjoint
// bit masks (order independent), the rest are plain stores.
//
// Workspace (caller owned, zero-filled once).  Header {ticket, done} plus one
// status word per partition.  Invariant: all zero between launches.  Each
// CTA increments `done` when its look-back is over; the CTA that brings it
// to the partition count (so no CTA can still be reading a status word)
// writes the arena offset / totals and zeroes the status words, the ticket
// and `done` for the next launch.
#include "common.cuh"

#include <mutex>

namespace bs {

#ifdef BS_PHASE_PROFILE
// Debug-only build: per-partition phase timestamps (globaltimer, ns).
constexpr int kProfParts = 1 << 16, kProfPhases = 10;
__device__ unsigned long long g_phase[kProfParts * kProfPhases];
__device__ __forceinline__ void phase_mark(long long part, int ph) {
  if (threadIdx.x == 0 && part >= 0 && part < kProfParts) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_phase[part * kProfPhases + ph] = t;
  }
}
#define PHASE(part, ph) phase_mark(part, ph)
#define PHASE_SYNC(part, ph) do { __syncthreads(); phase_mark(part, ph); } while (0)
#define PHASE_VAL(part, ph, v) do { if (threadIdx.x == 0 && part >= 0 && part < kProfParts) g_phase[(part) * kProfPhases + (ph)] = (v); } while (0)
#else
#define PHASE_VAL(part, ph, v) ((void)0)
#define PHASE(part, ph) ((void)0)
#define PHASE_SYNC(part, ph) ((void)0)
#endif

struct WsHeader {
  unsigned long long ticket;
  unsigned long long done;
  unsigned long long pad[14];
};

// status word: [63:62] state, [61:0] value
constexpr unsigned long long kAgg = 1ull << 62, kIncl = 2ull << 62;
constexpr unsigned long long kValMask = (1ull << 62) - 1;

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
  unsigned long long *flags;
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
// One chunk: load (32 B), optional quantisation, stored words + mask.
// ---------------------------------------------------------------------------
template <int DT_IN, bool QUANT, int TPP>
__device__ __forceinline__ uint32_t load_chunk(const CompressParams &P, int64_t grow,
                                               int64_t gcol, float qs,
                                               uint32_t (&sv)[Cfg<DT_IN, QUANT, TPP>::SW]) {
  using C = Cfg<DT_IN, QUANT, TPP>;
  uint32_t raw[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) raw[i] = 0;
  if (grow < P.M) {
    const uint8_t *src = P.dense + (grow * P.ld + gcol) * C::EB;
    if (P.vec_ok && gcol + C::VEC <= P.N) {
      asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                   : "=r"(raw[0]), "=r"(raw[1]), "=r"(raw[2]), "=r"(raw[3]), "=r"(raw[4]),
                     "=r"(raw[5]), "=r"(raw[6]), "=r"(raw[7])
                   : "l"(src));
    } else {
#pragma unroll
      for (int e = 0; e < C::VEC; ++e) {
        if (gcol + e < P.N) {
          uint32_t b;
          if constexpr (C::EB == 1) b = src[e];
          else if constexpr (C::EB == 2) b = reinterpret_cast<const uint16_t *>(src)[e];
          else b = reinterpret_cast<const uint32_t *>(src)[e];
          raw[e * C::EB / 4] |= b << (8 * ((e * C::EB) & 3));
        }
      }
    }
  }
  if constexpr (!QUANT) {
#pragma unroll
    for (int i = 0; i < 8; ++i) sv[i] = raw[i];
    return mask_of_words<C::SDT, 8>(raw);
  } else {
#pragma unroll
    for (int i = 0; i < C::SW; ++i) sv[i] = 0;
#pragma unroll
    for (int e = 0; e < C::VEC; ++e) {
      uint32_t b;
      if constexpr (C::EB == 2) b = (raw[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
      else b = raw[e];
      const float x = (DT_IN == BS_BF16) ? bf16_bits_to_f32(b) : __uint_as_float(b);
      float y = __fdiv_rn(x, qs);
      if constexpr (DT_IN == BS_BF16) y = bf16_bits_to_f32(f32_to_bf16_bits(y));
      sv[e >> 2] |= f32_to_e4m3_bits(y) << (8 * (e & 3));
    }
    if (P.qout && grow < P.M) {
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

__device__ __forceinline__ unsigned long long ld_rlx_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_rlx_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Block-wide min / sum (every thread calls; every thread gets the result).
__device__ __forceinline__ int block_min_int(int v, int *s_red) {
  v = __reduce_min_sync(0xFFFFFFFFu, v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  int r = s_red[0];
#pragma unroll
  for (int i = 1; i < kThreads / 32; ++i) r = min(r, s_red[i]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v,
                                                            unsigned long long *s_red) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, d);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  unsigned long long r = 0;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) r += s_red[i];
  __syncthreads();
  return r;
}

// MODE 0: fused single pass (look-back scan, writes bitmask + prefix + vals).
// MODE 1: compact only -- partition bases come from a given prefix[] (the
//         reference's compact_vals); bitmask / prefix are not written.
// MODE 2: tile_pack only -- bitmask + per-tile counts, no scan, no values.
template <int DT_IN, bool QUANT, bool PACK, int TPP, int MODE>
__global__ void __launch_bounds__(kThreads)
compress_kernel(const CompressParams P) {
  using C = Cfg<DT_IN, QUANT, TPP>;
  constexpr int NW = C::S * 8;  // warp-total slots
  extern __shared__ __align__(128) uint8_t smem_dyn[];
  __shared__ uint32_t s_wt[NW];
  __shared__ uint32_t s_tile_incl[TPP];
  __shared__ long long s_part;
  __shared__ long long s_off0;
  __shared__ long long s_excl;
  __shared__ uint32_t s_total;
  __shared__ int s_clean;
  __shared__ int s_red_i[kThreads / 32];
  __shared__ unsigned long long s_red_u[kThreads / 32];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid == 0) {
    long long part = blockIdx.x;
    if (MODE == 0) part = (long long)atomicAdd(&P.hdr->ticket, 1ull);
    s_part = part;
    long long off = 0;
    if (P.arena_offset) {
      off = *(volatile long long *)P.arena_offset;
      if (PACK && MODE == 0) off = (off + 7) / 8 * 8;  // functions.py:78-81
    }
    s_off0 = off;
    s_clean = 0;
  }
  __syncthreads();
  const long long part = s_part;
  const float qs = QUANT ? *P.qscale : 1.f;
  if (MODE == 0) PHASE(part, 0);

  // ---- load + mask ---------------------------------------------------------
  uint32_t sv[C::S][C::SW];
  uint32_t msk[C::S];
#pragma unroll
  for (int s = 0; s < C::S; ++s) {
    const int c = s * kThreads + tid;
    const int j = c / C::CPT, cc = c % C::CPT;
    const long long tile = part * TPP + j;
    if (tile < P.num_tiles) {
      const long long tm = tile / P.grid_n, tn = tile % P.grid_n;
      const int row = cc / C::CPR, colc = cc % C::CPR;
      msk[s] = load_chunk<DT_IN, QUANT, TPP>(P, tm * kTileM + row, tn * kTileN + colc * C::VEC,
                                             qs, sv[s]);
      if (MODE != 1) {
        uint8_t *bm = P.bitmask + tile * kTileBytes + cc * (C::VEC / 8);
        if constexpr (C::VEC == 8) *bm = (uint8_t)msk[s];
        else if constexpr (C::VEC == 16) *reinterpret_cast<uint16_t *>(bm) = (uint16_t)msk[s];
        else *reinterpret_cast<uint32_t *>(bm) = msk[s];
      }
    } else {
      msk[s] = 0;
#pragma unroll
      for (int i = 0; i < C::SW; ++i) sv[s][i] = 0;
    }
  }

  // ---- block scan of chunk counts in (slot, warp, lane) order ---------------
  uint32_t lex[C::S];
  if (MODE == 0) PHASE_SYNC(part, 1);
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
    if (lane == 0) s_total = carry;
  }
  __syncthreads();
  const uint32_t total = s_total;
  if (tid < TPP) {
    // chunk (tid+1)*CPT starts tile tid+1; its warp slot is that index / 32
    const int nxt = (tid + 1) * C::CPT / 32;
    s_tile_incl[tid] = nxt < NW ? s_wt[nxt] : total;
  }
  __syncthreads();

  if (MODE == 2) {
    if (tid < TPP && part * TPP + tid < P.num_tiles)
      P.counts[part * TPP + tid] =
          (int32_t)(s_tile_incl[tid] - (tid ? s_tile_incl[tid - 1] : 0u));
    return;
  }

  // ---- partition offset: block-wide decoupled look-back --------------------
  if (MODE == 0) {
    PHASE(part, 2);
    unsigned long long *F = P.flags;
    if (tid == 0) st_rlx_u64(&F[part], (part == 0 ? kIncl : kAgg) | total);
    long long excl = 0;
    if (part > 0) {
      long long idx = part - 1;
      uint32_t polls = 0;
      while (true) {
        const long long q = idx - tid;
        unsigned long long w = kIncl;  // before partition 0: inclusive 0
        if (q >= 0) w = ld_rlx_u64(&F[q]);
        const unsigned long long st = w & ~kValMask;
        const int first_incl = block_min_int(st == kIncl ? tid : kThreads, s_red_i);
        const int first_empty = block_min_int(st == 0 ? tid : kThreads, s_red_i);
        if (first_empty < kThreads && first_empty <= first_incl) {
          if (++polls > kMaxPolls) {  // give up: record it, do not hang
            if (tid == 0) status_or(P.status, BS_STATUS_TIMEOUT);
            break;
          }
          __nanosleep(64);
          continue;
        }
        const unsigned long long contrib = (tid <= first_incl) ? (w & kValMask) : 0ull;
        excl += (long long)block_sum_u64(contrib, s_red_u);
        if (first_incl < kThreads) break;
        idx -= kThreads;
      }
      PHASE(part, 6);
      PHASE_VAL(part, 8, polls);
      PHASE_VAL(part, 9, (unsigned long long)(part - 1 - idx) / kThreads + 1);
      if (tid == 0) st_rlx_u64(&F[part], kIncl | ((unsigned long long)excl + total));
    }
    if (tid == 0) {
      s_excl = excl;
      if (part == 0) P.prefix[0] = 0;
      __threadfence();
      const unsigned long long d = atomicAdd(&P.hdr->done, 1ull) + 1;
      PHASE(part, 7);
      if (d == (unsigned long long)P.num_parts) {
        // Last CTA out of its look-back: every CTA has read the arena
        // offset and no CTA reads a status word any more.
        __threadfence();
        const long long nnz = (long long)(ld_rlx_u64(&F[P.num_parts - 1]) & kValMask);
        if (P.arena_offset) *P.arena_offset = s_off0 + nnz;
        if (P.vals_offset_out) *P.vals_offset_out = s_off0;
        if (P.nnz_out) *P.nnz_out = nnz;
        s_clean = 1;
      }
    }
  } else {
    if (tid == 0) s_excl = (long long)P.prefix[part * TPP];
  }
  __syncthreads();
  const long long excl = s_excl;
  if (MODE == 0) PHASE(part, 3);
  if (MODE == 0) {
    if (s_clean) {  // zero the status words, the ticket and done
      for (long long i = tid; i < P.num_parts; i += kThreads) st_rlx_u64(&P.flags[i], 0ull);
      if (tid == 0) {
        P.hdr->ticket = 0;
        P.hdr->done = 0;
      }
    }
    if (tid < TPP && part * TPP + tid < P.num_tiles)
      P.prefix[part * TPP + tid + 1] = (uint32_t)(excl + s_tile_incl[tid]);
  }
  if (P.vals == nullptr) return;

  // ---- values ----------------------------------------------------------------
  const long long gbase = s_off0 + excl;  // logical index of first value
  const long long n = total;
  uint8_t *stage = smem_dyn;
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
  if (MODE == 0) PHASE(part, 4);

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
    if (MODE == 0) PHASE_SYNC(part, 5);
  } else {
    constexpr int B = C::BITS;
    const long long bit0 = gbase * B;
    const long long bit1 = (gbase + n) * B;
    const bool last = (part == P.num_parts - 1);
    const long long cap_words = P.cap / 4;
    // Standalone stream: the last partition owns (and zeroes) the bits after
    // the payload up to the end of packed_storage_nbytes(nnz) (payload
    // rounded to a word, plus one guard word; bitpacking.py:32-34).
    long long own_end = bit1;
    if (MODE == 0 && last && P.arena_offset == nullptr) {
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
      long long k = rel > 0 ? rel / B : 0;
      for (; k < n; ++k) {
        const long long sb = bit0 + k * B - wb;  // start of value k rel. to word
        if (sb >= 32) break;
        uint32_t v;
        if constexpr (C::SB == 1) v = stage[k];
        else v = reinterpret_cast<const uint16_t *>(stage)[k];
        v &= (1u << B) - 1u;
        acc |= (unsigned long long)v << (sb + 32);  // sb > -B >= -15
      }
      const uint32_t val = (uint32_t)(acc >> 32);
      const long long lo = bit0 > wb ? bit0 - wb : 0;
      const long long hi = own_end < wb + 32 ? own_end - wb : 32;
      const uint32_t own = (hi >= 32 ? 0xFFFFFFFFu : ((1u << hi) - 1u)) & ~((1u << lo) - 1u);
      merge_word(words + w, val, own);
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Tiles per partition.  MODE 0 wants big partitions (fewer look-back rounds
// per byte); 1-byte inputs need an even count (128 chunks per tile).
constexpr int tpp_for(int eb, int mode) { return mode == 0 ? 4 : (eb == 1 ? 2 : 1); }

template <int DT_IN, bool QUANT, bool PACK, int MODE>
static int launch_t(const CompressParams &P, cudaStream_t st) {
  constexpr int TPP = tpp_for(Elt<DT_IN>::bytes, MODE);
  using C = Cfg<DT_IN, QUANT, TPP>;
  constexpr size_t smem = (MODE == 2) ? 0 : (size_t)TPP * kTileNumel * C::SB + 16;
  static_assert(smem <= 48 * 1024, "stage fits the default dynamic shared memory");
  compress_kernel<DT_IN, QUANT, PACK, TPP, MODE><<<(unsigned)P.num_parts, kThreads, smem, st>>>(P);
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
  // One status word per partition; a partition is never smaller than a tile.
  return sizeof(WsHeader) + (size_t)num_tiles * sizeof(unsigned long long);
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
  P.flags = reinterpret_cast<unsigned long long *>(static_cast<uint8_t *>(workspace) +
                                                   sizeof(WsHeader));
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

#ifdef BS_PHASE_PROFILE
extern "C" int bs_debug_phases(unsigned long long *host_out) {
  return cudaMemcpyFromSymbol(host_out, bs::g_phase, sizeof(bs::g_phase)) == cudaSuccess ? 0 : 5;
}
#endif

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
