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
// consecutive tiles (tile id order = output order).  Partitions are handed
// out by an atomic ticket, so partition p is only ever processed by a CTA
// that started after the CTAs of partitions < p: the decoupled look-back
// below therefore only waits on CTAs that are already running.
//
// Per tile, the 4096 elements are split into 16-byte (32 for fp32 input)
// chunks of VEC = 8 or 16 consecutive row elements; thread i owns chunks
// i, i+256, ... .  A warp's load covers whole 128/64-byte tile rows, so every
// DRAM sector is used in full.  Each chunk yields VEC mask bits, which are
// exactly the chunk's bitmask byte (VEC = 8) or 16-bit half-word (VEC = 16)
// in the reference's LSB-first, row-major-in-tile bit order.
//
// Offsets.  A block-wide exclusive scan of chunk popcounts in (tile, chunk)
// order gives each chunk's value offset inside the partition; the partition
// total is published to the scan workspace and a warp looks back over the
// predecessors' flags (single-pass scan with decoupled look-back) to get the
// partition's global offset.  Every wait is bounded (kMaxPolls); on expiry
// the CTA records BS_STATUS_TIMEOUT and carries on, so no CTA spins forever.
//
// Values.  Raw storage: the partition's values are staged in shared memory
// already shifted by the destination's misalignment, then written with
// aligned 16-byte stores (element stores only on the two edge vectors, which
// neighbouring partitions share).  Packed storage (15/7-bit): the staged
// values are re-packed into 32-bit words of the continuous bitstream; words
// that a neighbouring partition also writes are merged with atomicAnd /
// atomicOr on disjoint bit masks (order independent), the rest are stored.
//
// Workspace (caller owned, zero-filled once): a header {ticket, launch_base}
// and one flag record per partition {tag, aggregate, inclusive}.  tag =
// launch_base * 4 + state, where launch_base (the ticket count before this
// launch) is unique per launch, so flags left by earlier launches never
// match.  The CTA of the last partition writes launch_base += grid after the
// scan is complete -- by then every CTA has read it (each reads it before
// publishing, and the last look-back transitively observed every publish).
#include "common.cuh"

namespace bs {

struct WsHeader {
  unsigned long long ticket;
  unsigned long long launch_base;
  unsigned long long pad[14];
};
struct ScanFlag {
  unsigned long long tag;
  unsigned long long agg;
  unsigned long long incl;
  unsigned long long pad;
};
constexpr int kStateAgg = 1, kStateIncl = 2;

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
  ScanFlag *flags;
  int32_t *status;
  int64_t grid_n, num_tiles, num_parts;
  int vec_ok;    // dense base and row stride allow 16-byte vector loads
  int vals_v16;  // vals base 16-byte aligned (raw storage)
  int qout_v8;   // quant_out rows allow 8-byte stores
};

template <int DT_IN, bool QUANT>
struct Cfg {
  static constexpr int SDT = QUANT ? BS_E4M3 : DT_IN;      // stored dtype
  static constexpr int EB = Elt<DT_IN>::bytes;              // input bytes
  static constexpr int SB = Elt<SDT>::bytes;                // stored bytes
  static constexpr int VEC = (EB == 1) ? 16 : 8;            // elements / chunk
  static constexpr int CPR = kTileN / VEC;                  // chunks / tile row
  static constexpr int CPT = kTileNumel / VEC;              // chunks / tile
  static constexpr int CH = CPT / kThreads;                 // chunks / thread
  static constexpr int LW = VEC * EB / 16;                  // uint4 loads / chunk
  static constexpr int SW = VEC * SB / 4;                   // u32 words stored
  static constexpr int EPV = 16 / SB;                       // stored elts / 16B
  static constexpr int BITS = pack_bits<SDT>();
};

// Load one chunk (VEC elements) and turn it into stored bits + a mask.
template <int DT_IN, bool QUANT>
__device__ __forceinline__ uint32_t load_chunk(const CompressParams &P, int64_t grow,
                                               int64_t gcol, float qs,
                                               uint32_t (&sv)[Cfg<DT_IN, QUANT>::SW]) {
  using C = Cfg<DT_IN, QUANT>;
  uint32_t raw[C::VEC * C::EB / 4];
#pragma unroll
  for (int i = 0; i < C::VEC * C::EB / 4; ++i) raw[i] = 0;
  if (grow < P.M) {
    const uint8_t *src = P.dense + (grow * P.ld + gcol) * C::EB;
    if (P.vec_ok && gcol + C::VEC <= P.N) {
#pragma unroll
      for (int l = 0; l < C::LW; ++l) {
        uint4 v = ld_nc_v4(src + 16 * l);
        raw[4 * l + 0] = v.x; raw[4 * l + 1] = v.y;
        raw[4 * l + 2] = v.z; raw[4 * l + 3] = v.w;
      }
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
  uint32_t mask = 0;
#pragma unroll
  for (int i = 0; i < C::SW; ++i) sv[i] = 0;
#pragma unroll
  for (int e = 0; e < C::VEC; ++e) {
    uint32_t b;
    if constexpr (C::EB == 1) b = (raw[e >> 2] >> (8 * (e & 3))) & 0xFFu;
    else if constexpr (C::EB == 2) b = (raw[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
    else b = raw[e];
    uint32_t s;
    if constexpr (QUANT) {
      float x = (DT_IN == BS_BF16) ? bf16_bits_to_f32(b) : __uint_as_float(b);
      float y = __fdiv_rn(x, qs);
      if constexpr (DT_IN == BS_BF16) y = bf16_bits_to_f32(f32_to_bf16_bits(y));
      s = f32_to_e4m3_bits(y);
    } else {
      s = b;
    }
    mask |= (uint32_t)is_pos<C::SDT>(s) << e;
    if constexpr (C::SB == 1) sv[e >> 2] |= s << (8 * (e & 3));
    else sv[e >> 1] |= s << (16 * (e & 1));
  }
  if constexpr (QUANT) {
    if (P.qout && grow < P.M) {
      uint8_t *dst = P.qout + grow * P.N + gcol;
      if (P.qout_v8 && gcol + C::VEC <= P.N) {
        if constexpr (C::VEC == 8) {
          *reinterpret_cast<uint2 *>(dst) = make_uint2(sv[0], sv[1]);
        } else {
          *reinterpret_cast<uint4 *>(dst) = make_uint4(sv[0], sv[1], sv[2], sv[3]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < C::VEC; ++e)
          if (gcol + e < P.N) dst[e] = (sv[e >> 2] >> (8 * (e & 3))) & 0xFFu;
      }
    }
  }
  return mask;
}

template <int SB>
__device__ __forceinline__ uint32_t get_elt(const uint32_t *sv, int e) {
  if constexpr (SB == 1) return (sv[e >> 2] >> (8 * (e & 3))) & 0xFFu;
  else return (sv[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
}

// Write bit range [own_lo, own_hi) of word w (other bits untouched).
__device__ __forceinline__ void merge_word(uint32_t *dst, uint32_t val, uint32_t own) {
  if (own == 0xFFFFFFFFu) {
    *dst = val;
  } else if (own) {
    atomicAnd(dst, ~own);
    atomicOr(dst, val & own);
  }
}

// MODE 0: fused single pass (look-back scan, writes bitmask + prefix + vals).
// MODE 1: compact only -- partition bases come from a given prefix[] (the
//         reference's compact_vals); bitmask / prefix are not written.
// MODE 2: tile_pack only -- bitmask + per-tile counts, no scan, no values.
template <int DT_IN, bool QUANT, bool PACK, int TPP, int MODE>
__global__ void __launch_bounds__(kThreads)
compress_kernel(const CompressParams P) {
  using C = Cfg<DT_IN, QUANT>;
  constexpr int NW = TPP * C::CH * 8;  // warp-total slots
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  __shared__ uint32_t s_wt[NW];
  __shared__ uint32_t s_tile_incl[TPP];
  __shared__ long long s_part;
  __shared__ unsigned long long s_base;  // launch base
  __shared__ long long s_off0;           // arena / stream start (values)
  __shared__ long long s_excl;           // partition's exclusive value offset
  __shared__ uint32_t s_total;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid == 0) {
    long long part;
    if (MODE == 0) {
      const unsigned long long t = atomicAdd(&P.hdr->ticket, 1ull);
      unsigned long long base =
          ld_relaxed_u64(&P.hdr->launch_base);
      part = (long long)(t - base);
      s_base = base;
    } else {
      part = blockIdx.x;
      s_base = 0;
    }
    s_part = part;
    long long off = 0;
    if (P.arena_offset) {
      off = *(volatile long long *)P.arena_offset;
      if (PACK && MODE == 0) off = (off + 7) / 8 * 8;  // functions.py:78-81
    }
    s_off0 = off;
  }
  __syncthreads();
  const long long part = s_part;
  if (part < 0 || part >= P.num_parts) {  // cannot happen with a sane workspace
    if (tid == 0) status_or(P.status, BS_STATUS_TIMEOUT);
    return;
  }
  const float qs = QUANT ? *P.qscale : 1.f;

  // ---- load + mask ---------------------------------------------------------
  uint32_t sv[TPP][C::CH][C::SW];
  uint32_t msk[TPP][C::CH];
  uint32_t cnt[TPP][C::CH];
#pragma unroll
  for (int j = 0; j < TPP; ++j) {
    const long long tile = part * TPP + j;
    const bool valid = tile < P.num_tiles;
    const long long tm = valid ? tile / P.grid_n : 0, tn = valid ? tile % P.grid_n : 0;
#pragma unroll
    for (int s = 0; s < C::CH; ++s) {
      const int c = s * kThreads + tid;
      const int row = c / C::CPR, cc = c % C::CPR;
      if (valid) {
        msk[j][s] = load_chunk<DT_IN, QUANT>(P, tm * kTileM + row, tn * kTileN + cc * C::VEC,
                                             qs, sv[j][s]);
      } else {
        msk[j][s] = 0;
#pragma unroll
        for (int i = 0; i < C::SW; ++i) sv[j][s][i] = 0;
      }
      cnt[j][s] = __popc(msk[j][s]);
      if (MODE != 1 && valid) {
        uint8_t *bm = P.bitmask + tile * kTileBytes;
        if constexpr (C::VEC == 8) bm[c] = (uint8_t)msk[j][s];
        else reinterpret_cast<uint16_t *>(bm)[c] = (uint16_t)msk[j][s];
      }
    }
  }

  // ---- block scan of chunk counts in (tile, slot, warp, lane) order ---------
  uint32_t lex[TPP][C::CH];
#pragma unroll
  for (int j = 0; j < TPP; ++j)
#pragma unroll
    for (int s = 0; s < C::CH; ++s) {
      uint32_t inc = warp_incl_scan(cnt[j][s]);
      lex[j][s] = inc - cnt[j][s];
      if (lane == 31) s_wt[(j * C::CH + s) * 8 + warp] = inc;
    }
  __syncthreads();
  if (warp == 0) {
    uint32_t carry = 0;
#pragma unroll
    for (int w0 = 0; w0 < NW; w0 += 32) {
      const int idx = w0 + lane;
      uint32_t v = idx < NW ? s_wt[idx] : 0;
      uint32_t inc = warp_incl_scan(v) + carry;
      if (idx < NW) s_wt[idx] = inc - v;
      carry = __shfl_sync(0xFFFFFFFFu, inc, 31);
    }
    if (lane == 0) s_total = carry;
  }
  __syncthreads();
  const uint32_t total = s_total;
  if (tid < TPP) {
    const int nxt = (tid + 1) * C::CH * 8;
    s_tile_incl[tid] = nxt < NW ? s_wt[nxt] : total;
  }

  if (MODE == 2) {
    __syncthreads();
    if (tid < TPP && part * TPP + tid < P.num_tiles)
      P.counts[part * TPP + tid] = (int32_t)(s_tile_incl[tid] - (tid ? s_tile_incl[tid - 1] : 0u));
    return;
  }

  // ---- partition offset ------------------------------------------------------
  if (MODE == 0) {
    if (warp == 0) {
      ScanFlag *F = P.flags;
      const unsigned long long E = s_base << 2;
      long long excl = 0;
      if (lane == 0) {
        if (part == 0) {
          F[0].incl = total;
          st_release_u64(&F[0].tag, E | kStateIncl);
        } else {
          F[part].agg = total;
          st_release_u64(&F[part].tag, E | kStateAgg);
        }
      }
      if (part > 0) {
        long long idx = part - 1;
        uint32_t polls = 0;
        bool timed_out = false;
        while (true) {
          const long long q = idx - lane;
          int state = kStateIncl;
          unsigned long long val = 0;
          if (q >= 0) {
            unsigned long long tag = ld_acquire_u64(&F[q].tag);
            state = ((tag & ~3ull) == E) ? (int)(tag & 3ull) : 0;
            if (state == kStateIncl) val = ld_relaxed_u64(&F[q].incl);
            else if (state == kStateAgg) val = ld_relaxed_u64(&F[q].agg);
          }
          if (__any_sync(0xFFFFFFFFu, state == 0)) {
            if (++polls > kMaxPolls) { timed_out = true; break; }
            __nanosleep(32);
            continue;
          }
          const uint32_t inc_mask = __ballot_sync(0xFFFFFFFFu, state == kStateIncl);
          const int stop = inc_mask ? (__ffs(inc_mask) - 1) : 31;
          unsigned long long contrib = (lane <= stop) ? val : 0ull;
#pragma unroll
          for (int d = 16; d > 0; d >>= 1) contrib += __shfl_xor_sync(0xFFFFFFFFu, contrib, d);
          excl += (long long)contrib;
          if (inc_mask) break;
          idx -= 32;
        }
        if (timed_out && lane == 0) status_or(P.status, BS_STATUS_TIMEOUT);
        if (lane == 0) {
          F[part].incl = (unsigned long long)excl + total;
          st_release_u64(&F[part].tag, E | kStateIncl);
        }
      }
      if (lane == 0) {
        s_excl = excl;
        if (part == P.num_parts - 1) {
          const long long nnz = excl + (long long)total;
          // Every CTA of this launch has read launch_base and arena_offset.
          P.hdr->launch_base = s_base + (unsigned long long)P.num_parts;
          if (P.arena_offset) *P.arena_offset = s_off0 + nnz;
          if (P.vals_offset_out) *P.vals_offset_out = s_off0;
          if (P.nnz_out) *P.nnz_out = nnz;
        }
        if (part == 0) P.prefix[0] = 0;
      }
    }
  } else {
    if (tid == 0) s_excl = (long long)P.prefix[part * TPP];
  }
  __syncthreads();
  const long long excl = s_excl;
  if (MODE == 0 && tid < TPP && part * TPP + tid < P.num_tiles)
    P.prefix[part * TPP + tid + 1] = (uint32_t)(excl + s_tile_incl[tid]);
  if (P.vals == nullptr) return;

  // ---- values ----------------------------------------------------------------
  const long long gbase = s_off0 + excl;  // logical index of first value
  const long long n = total;
  uint8_t *stage = smem_dyn;
  const int shift = PACK ? 0 : (int)(gbase % C::EPV);
#pragma unroll
  for (int j = 0; j < TPP; ++j)
#pragma unroll
    for (int s = 0; s < C::CH; ++s) {
      const uint32_t m = msk[j][s];
      uint32_t k = shift + s_wt[(j * C::CH + s) * 8 + warp] + lex[j][s];
#pragma unroll
      for (int e = 0; e < C::VEC; ++e) {  // static indices keep sv in registers
        if ((m >> e) & 1u) {
          const uint32_t v = get_elt<C::SB>(sv[j][s], e);
          if constexpr (C::SB == 1) stage[k] = (uint8_t)v;
          else reinterpret_cast<uint16_t *>(stage)[k] = (uint16_t)v;
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
    long long bit1 = (gbase + n) * B;
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
      long long rel = wb - bit0;  // bit offset of word start inside our range
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
template <int DT_IN, bool QUANT, bool PACK, int TPP, int MODE>
static int launch_t(const CompressParams &P, cudaStream_t st) {
  using C = Cfg<DT_IN, QUANT>;
  const size_t smem = (size_t)TPP * kTileNumel * C::SB + 16;
  static_assert((size_t)TPP * kTileNumel * C::SB + 16 <= 48 * 1024,
                "stage must fit the default dynamic shared memory limit");
  auto k = compress_kernel<DT_IN, QUANT, PACK, TPP, MODE>;
  k<<<(unsigned)P.num_parts, kThreads, smem, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? BS_OK : BS_ERR_LAUNCH;
}

template <int DT_IN, bool QUANT, int MODE>
static int launch_pack(const CompressParams &P, int pack, int tpp, cudaStream_t st) {
  if (pack) {
    if (tpp == 1) return launch_t<DT_IN, QUANT, true, 1, MODE>(P, st);
    return launch_t<DT_IN, QUANT, true, 2, MODE>(P, st);
  }
  if (tpp == 1) return launch_t<DT_IN, QUANT, false, 1, MODE>(P, st);
  return launch_t<DT_IN, QUANT, false, 2, MODE>(P, st);
}

template <int MODE>
static int dispatch(const CompressParams &P, int dt, bool quant, int pack, int tpp,
                    cudaStream_t st) {
  if (quant) {
    if (dt == BS_BF16) return launch_pack<BS_BF16, true, MODE>(P, pack, tpp, st);
    if (dt == BS_F32) return launch_pack<BS_F32, true, MODE>(P, pack, tpp, st);
    return BS_ERR_DTYPE;
  }
  switch (dt) {
    case BS_BF16: return launch_pack<BS_BF16, false, MODE>(P, pack, tpp, st);
    case BS_E4M3: return launch_pack<BS_E4M3, false, MODE>(P, pack, tpp, st);
    case BS_E5M2: return launch_pack<BS_E5M2, false, MODE>(P, pack, tpp, st);
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

// Tiles per partition: 2 once there are enough partitions to fill the GPU
// several times over, else 1 (more, smaller CTAs for small tensors).
static int pick_tpp(int64_t num_tiles) { return num_tiles >= 148 * 8 ? 2 : 1; }

static int fill_common(CompressParams &P, const void *dense, int dt, int64_t M, int64_t N,
                       int64_t ld) {
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
  P.vec_ok = ((reinterpret_cast<uintptr_t>(dense) & 15) == 0) && ((ld * eb) % 16 == 0);
  return BS_OK;
}

}  // namespace bs

using namespace bs;

extern "C" size_t bs_compress_workspace_bytes(int64_t num_tiles) {
  if (num_tiles < 0) num_tiles = 0;
  return sizeof(WsHeader) + (size_t)num_tiles * sizeof(ScanFlag);
}

extern "C" int bs_compress(const void *dense, int in_dtype, int64_t M, int64_t N, int64_t ld,
                           const float *quant_scale, uint8_t *quant_out, uint8_t *bitmask,
                           uint32_t *prefix, void *vals, int64_t vals_capacity, int pack_sbit,
                           int64_t *arena_offset, int64_t *vals_offset_out, int64_t *nnz_out,
                           void *workspace, size_t workspace_bytes, int32_t *status,
                           void *stream) {
  CompressParams P{};
  int rc = fill_common(P, dense, in_dtype, M, N, ld);
  if (rc) return rc;
  const bool quant = quant_scale != nullptr;
  if (quant && in_dtype != BS_BF16 && in_dtype != BS_F32) return BS_ERR_DTYPE;
  if (!quant && in_dtype == BS_F32) return BS_ERR_DTYPE;
  if (!bitmask || !prefix || !workspace) return BS_ERR_ARG;
  if (pack_sbit != 0 && pack_sbit != 1) return BS_ERR_ARG;
  if (vals_capacity < 0) return BS_ERR_CAPACITY;
  if (pack_sbit && vals && (reinterpret_cast<uintptr_t>(vals) & 3)) return BS_ERR_ALIGN;
  if (pack_sbit && (vals_capacity & 3)) return BS_ERR_ALIGN;
  const int tpp = pick_tpp(P.num_tiles);
  P.num_parts = (P.num_tiles + tpp - 1) / tpp;
  if (workspace_bytes < bs_compress_workspace_bytes(P.num_parts)) return BS_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 15) return BS_ERR_ALIGN;
  P.qscale = quant_scale;
  P.qout = quant_out;
  P.qout_v8 = quant_out && ((reinterpret_cast<uintptr_t>(quant_out) & 15) == 0) &&
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
  P.flags = reinterpret_cast<ScanFlag *>(static_cast<uint8_t *>(workspace) + sizeof(WsHeader));
  P.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (P.num_tiles == 0) {
    // Empty tensor: prefix = [0], offsets as if nnz = 0.
    if (cudaMemsetAsync(prefix, 0, sizeof(uint32_t), st) != cudaSuccess) return BS_ERR_LAUNCH;
    return BS_OK;  // arena offset unchanged; vals_offset_out / nnz_out untouched
  }
  return dispatch<0>(P, in_dtype, quant, pack_sbit, tpp, st);
}

// Reference compact_vals (lib_sparse/src/triton_operators.py:36-115): values
// only, bases from an existing prefix.  `vals_offset` is a device int64*
// holding the logical start (may be NULL for 0).
extern "C" int bs_compact_vals(const void *dense, int dtype, int64_t M, int64_t N, int64_t ld,
                               const uint32_t *prefix, void *vals, int64_t vals_capacity,
                               int pack_sbit, const int64_t *vals_offset, int32_t *status,
                               void *stream) {
  CompressParams P{};
  int rc = fill_common(P, dense, dtype, M, N, ld);
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
  P.num_parts = P.num_tiles;
  if (P.num_tiles == 0) return BS_OK;
  return dispatch<1>(P, dtype, false, pack_sbit, 1, static_cast<cudaStream_t>(stream));
}

extern "C" int bs_tile_pack(const void *dense, int dtype, int64_t M, int64_t N, int64_t ld,
                            int32_t *counts, uint8_t *bitmask, void *stream) {
  CompressParams P{};
  int rc = fill_common(P, dense, dtype, M, N, ld);
  if (rc) return rc;
  if (dtype == BS_F32) return BS_ERR_DTYPE;
  if (P.num_tiles == 0) return BS_OK;
  if (!counts || !bitmask) return BS_ERR_ARG;
  P.counts = counts;
  P.bitmask = bitmask;
  P.num_parts = P.num_tiles;
  return dispatch<2>(P, dtype, false, 0, 1, static_cast<cudaStream_t>(stream));
}
