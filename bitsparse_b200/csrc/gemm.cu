// K3 -- tcgen05 GEMM with the ReLU mask fused into its epilogue.
//
//   C[M, N] = (A[M, K] . B[K, N]) (.) mask        (bf16 in, fp32 accumulate, bf16 out)
//
// A is row-major (K contiguous: "K-major"), B is row-major (N contiguous:
// "MN-major"), both read by TMA with the 128-byte swizzle into the layouts
// tcgen05.mma reads directly.  mask (optional) is the bitmask of a
// bitsparse [M, N] tensor (64 x 64 tiles, grid-row-major, LSB-first): an
// output element whose bit is clear is written as +0.  This is the
// backward of ReluLinear (lib_sparse/layers.py:38-51, gradient half of
// mask_with_bitmask_ in lib_sparse/src/triton_kernels.py:249-276):
// grad_z = (grad_y @ W) masked by h > 0, without the dense grad_h ever
// reaching HBM.
//
// Persistent: one CTA per SM walks a static schedule of 128 x 256 tiles of
// C (M tile = the 128 TMEM lanes, N tile = 256 fp32 TMEM columns), with two
// accumulators in TMEM (all 512 columns) so that the epilogue of one tile
// overlaps the main loop of the next:
//   warp 0      TMA producer: for each 64-wide K block of each tile, A box
//               [128 x 64] and four B boxes [64 x 64] into the next of 4
//               stages (48 KB);
//   warp 1      MMA issuer (one thread): four tcgen05.mma (K = 16 each) per
//               stage, tcgen05.commit to the stage's "empty" barrier, and
//               after a tile's last stage to that accumulator's "full"
//               barrier; it also allocates and frees the TMEM columns;
//   warps 2..5  epilogue: the row's bitmask words are fetched before the
//               wait; tcgen05.ld of 64 columns at a time from the warp's
//               TMEM lane quarter (warp % 4), bf16 rounding, masking, a
//               swizzled 32 x 64 staging box in shared memory (two per warp,
//               alternating) and a TMA store of the box (clipped at the
//               edges); then the accumulator is handed back to the MMA warp.
// All mbarrier waits are bounded (BS_STATUS_TIMEOUT); the producer waits
// for its own copies before the CTA exits; TMEM is always freed.
#include "common.cuh"

#include <cuda.h>  // CUtensorMap (types only; the encoder comes through the runtime)

#include <cstdlib>
#include <mutex>

namespace bs {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kThreadsG = 192;  // 6 warps
constexpr uint32_t kTmemCols = 256;
// Epilogue staging: per epilogue warp two 32-row x 64-column bf16 boxes
// (128-byte rows, 128-byte swizzle) for the TMA stores of C.
constexpr int kEpiBox = 32 * 64 * 2;  // 4 KB
constexpr int kEpiBytes = 4 * 2 * kEpiBox;

struct GemmParams {
  uint8_t *C;
  int64_t M, N, K, ldc;
  const uint8_t *mask;  // bitmask of a bitsparse [M, N] tensor, or null
  int64_t mask_grid_n;  // its tile columns: ceil(N / 64)
  int64_t mask_grid_m;  // its tile rows: ceil(M / 64)
  int c_tma;            // C is written by TMA stores (aligned base and row stride)
  int32_t *status;
  // ReLU^2 epilogue: the stored activation's raw bf16 values, tile prefix
  // and value offset, and 2k (RELU2_SCALE k)
  const uint16_t *vals;
  const uint32_t *prefix;
  const int64_t *vals_offset;
  float two_k;
  // FP8 form: the per-tensor scales of A and B (device fp32 scalars)
  const float *scale_a, *scale_b;
  // FP8 ReLU^2 epilogue: the stored activation's e4m3 scale, or null
  const float *hscale;
};

// Epilogues: none, the ReLU mask, the ReLU^2 gradient; kEpiFp8 is the FP8
// form of the GEMM (e4m3 operands, both K-major, C = bf16(acc * sa * sb)).
// kEpiFp8Relu2 is the FP8 GEMM with the ReLU^2 gradient of an e4m3-stored
// activation in its epilogue.
enum { kEpiNone = 0, kEpiMask = 1, kEpiRelu2 = 2, kEpiFp8 = 3, kEpiFp8Relu2 = 4 };
template <int EPI>
constexpr bool epi_f8() { return EPI == kEpiFp8 || EPI == kEpiFp8Relu2; }
template <int EPI>
constexpr bool epi_relu2() { return EPI == kEpiRelu2 || EPI == kEpiFp8Relu2; }
// K elements per stage: 64 bf16 or 128 e4m3 -- 128-byte rows either way
template <int EPI>
constexpr int stage_k() { return epi_f8<EPI>() ? 128 : kBK; }

__device__ __forceinline__ uint32_t saddr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// Bounded wait: false (and the status word flagged) if the phase never came.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int32_t *status) {
  for (uint32_t n = 0; n < kMaxPolls; ++n)
    if (mbar_try_wait(bar, parity)) return true;
  status_or(status, BS_STATUS_TIMEOUT);
  return false;
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(saddr(bar))
      : "memory");
}

// Shared-memory matrix descriptor (tcgen05): start address, leading and
// stride byte offsets (all >> 4), version 1, layout 2 = 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
template <int CG, bool F8 = false>
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  if constexpr (F8 && CG == 2)
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  else if constexpr (F8)
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  else if constexpr (CG == 2)
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
  else
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive on the barrier at shared::cluster address `bar` once every MMA
// issued so far by this thread has completed.
template <int CG>
__device__ __forceinline__ void mma_commit_to(uint32_t bar) {
  if constexpr (CG == 2)
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// TMA tile load of one CTA of a pair, completing on the barrier at
// shared::cluster address `bar` (the leader's).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int x, int y,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Two fp32 -> bf16 conversions, round to nearest even (the hardware
// conversion; it matches torch's bf16 rounding for every non-NaN value).
__device__ __forceinline__ uint32_t bf16x2_rn(uint32_t lo, uint32_t hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(hi)), "f"(__uint_as_float(lo)));
  return r;
}

// 32 consecutive fp32 columns of this thread's TMEM lane (no wait).
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}


// Tile t of the static schedule -> (m block, n block): groups of kGroupM
// row blocks sweep the column blocks together, so neighbouring CTAs share
// B columns and A rows in L2.
constexpr int kGroupM = 8;
__device__ __forceinline__ void tile_coords(int64_t t, int64_t mt, int64_t nt, int64_t &mb,
                                            int64_t &nb) {
  const int64_t per_group = (int64_t)kGroupM * nt;
  const int64_t g = t / per_group, first_m = g * kGroupM;
  const int64_t gm = mt - first_m < kGroupM ? mt - first_m : kGroupM;
  const int64_t r = t - g * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

// Per cluster size CG (1: one CTA per tile; 2: a CTA pair shares a
// 256 x 256 tile through tcgen05's cta_group::2, each CTA loading its 128
// rows of A and 128 of the 256 columns of B, so a stage is 32 KB instead
// of 48 KB and the operand bytes per flop drop by a third).
// ReLU^2 epilogue: per epilogue warp two staging buffers, each for the
// values of its 32 rows of one 64 x 64 tile (at most 2048 bf16, as the
// 16-byte aligned superset); chunk c + 2's values are copied in while chunk
// c is expanded.
constexpr int kValStage = 2048 * 2 + 32;
constexpr int kValBufs = 2;
template <int CG, int EPI = kEpiNone>
struct GemmCfg {
  static constexpr int BM = kBM * CG;           // rows of C per tile
  static constexpr int BNL = kBN / CG;          // columns of B this CTA loads
  static constexpr int BBYTES = kBK * BNL * 2;  // B bytes per stage and CTA
  static constexpr int STAGE = kABytes + BBYTES;
  // stages (one fewer with the ReLU^2 epilogue's value staging)
  static constexpr int NST = (CG == 2 ? 6 : 4) - (epi_relu2<EPI>() ? 1 : 0);
  static constexpr int VBYTES = epi_relu2<EPI>() ? 4 * kValBufs * kValStage + 512 : 0;
  static constexpr size_t SMEM = 1024 + (size_t)NST * STAGE + kEpiBytes + VBYTES + 256;
  // instruction descriptor: fp32 accumulator, M = BM, N = kBN; bf16 A
  // (K-major) and B (MN-major), or e4m3 A and B (both K-major)
  static constexpr uint32_t IDESC =
      epi_f8<EPI>()
          ? ((1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24))
          : ((1u << 4) | (1u << 7) | (1u << 10) | (0u << 15) | (1u << 16) |
             ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24));
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// 16-byte global -> shared copy (cp.async, completion per thread by group).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

template <int EPI, int CG>
__global__ void __launch_bounds__(kThreadsG, 1)
    gemm_mask_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const GemmParams P) {
  using G = GemmCfg<CG, EPI>;
  constexpr bool F8 = epi_f8<EPI>();
  constexpr bool RELU2 = epi_relu2<EPI>();
  constexpr bool MASK = EPI == kEpiMask || RELU2;
  constexpr int VB = EPI == kEpiFp8Relu2 ? 1 : 2;  // bytes per stored value
  constexpr int BKE = stage_k<EPI>();  // K elements per stage
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms (same offsets in both
  // CTAs of a pair, which the cta_group::2 descriptors rely on)
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *epi = smem + (size_t)G::NST * G::STAGE;  // staging boxes
  uint8_t *vstage = epi + kEpiBytes;                 // ReLU^2: value staging
  uint64_t *full = reinterpret_cast<uint64_t *>(vstage + G::VBYTES);
  uint64_t *empty = full + G::NST;
  uint64_t *acc_full = empty + G::NST;  // [2]: MMA -> epilogue
  uint64_t *acc_empty = acc_full + 2;   // [2]: epilogue -> MMA
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = CG == 2 ? cluster_rank() : 0;
  const bool leader = rank == 0;
  const int64_t cid = (int64_t)blockIdx.x / CG, ncl = (int64_t)gridDim.x / CG;
  const int nk = (int)((P.K + BKE - 1) / BKE);
  const int64_t mt = (P.M + G::BM - 1) / G::BM, nt = (P.N + kBN - 1) / kBN;
  const int64_t ntiles = mt * nt;

  // FP8 ReLU^2: bf16 bits of every e4m3 code (exact: e4m3 values are bf16
  // values), filled before the start-up barrier below
  uint16_t *code_bf16 = reinterpret_cast<uint16_t *>(vstage + 4 * kValBufs * kValStage);
  if constexpr (EPI == kEpiFp8Relu2) {
    for (int c = threadIdx.x; c < 256; c += blockDim.x)
      code_bf16[c] = (uint16_t)(__float_as_uint(store_bits_to_f32<BS_E4M3>((uint32_t)c)) >> 16);
  }
  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    for (int s = 0; s < G::NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4 * CG);  // one arrival per epilogue warp of the pair
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // the whole warp allocates (sync.aligned); both CTAs of a pair
    if constexpr (CG == 2) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       saddr(tmem_slot)),
                   "r"(2 * kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       saddr(tmem_slot)),
                   "r"(2 * kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync();  // both CTAs' barriers initialised
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int64_t it = 0;  // global k-block counter: stage it % NST, phase it / NST
      bool ok = true;
      // the stage's "full" barrier is the leader's; it expects both CTAs' bytes
      for (int64_t t = cid; t < ntiles && ok; t += ncl) {
        int64_t mb, nb;
        tile_coords(t, mt, nt, mb, nb);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = (int)(it % G::NST);
          if (it >= G::NST &&
              !mbar_wait(&empty[s], (uint32_t)((it / G::NST - 1) & 1), P.status)) {
            ok = false;
            break;
          }
          uint8_t *a = smem + (size_t)s * G::STAGE;
          uint8_t *b = a + kABytes;
          const int ay = (int)(mb * G::BM + rank * kBM);
          const int bx = (int)(nb * kBN + rank * G::BNL);
          if constexpr (CG == 2) {
            if (leader) mbar_expect_tx(&full[s], 2 * G::STAGE);
            const uint32_t bar = map_rank(saddr(&full[s]), 0);
            tma_load_2d_pair(a, &tmA, kb * BKE, ay, bar);
#pragma unroll
            for (int j = 0; j < G::BNL / 64; ++j) {
              if constexpr (F8)  // B^T rows (K-major): 64 rows of 128 K-bytes per box
                tma_load_2d_pair(b + j * 8192, &tmB, kb * BKE, bx + 64 * j, bar);
              else
                tma_load_2d_pair(b + j * 8192, &tmB, bx + 64 * j, kb * BKE, bar);
            }
          } else {
            mbar_expect_tx(&full[s], G::STAGE);
            tma_load_2d(a, &tmA, kb * BKE, ay, &full[s]);
#pragma unroll
            for (int j = 0; j < G::BNL / 64; ++j) {
              if constexpr (F8)
                tma_load_2d(b + j * 8192, &tmB, kb * BKE, bx + 64 * j, &full[s]);
              else
                tma_load_2d(b + j * 8192, &tmB, bx + 64 * j, kb * BKE, &full[s]);
            }
          }
        }
      }
      // every copy landed before the CTA may exit (the leader's barriers
      // count the peer's copies too)
      if (leader)
        for (int64_t i = it - G::NST < 0 ? 0 : it - G::NST; i < it; ++i)
          mbar_wait(&full[i % G::NST], (uint32_t)((i / G::NST) & 1), P.status);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int64_t it = 0;
      int j = 0;  // local tile counter: accumulator buffer j & 1, use j >> 1
      bool ok = true;
      for (int64_t t = cid; t < ntiles && ok; t += ncl, ++j) {
        const int buf = j & 1;
        if (j >= 2 && !mbar_wait(&acc_empty[buf], (uint32_t)(((j >> 1) - 1) & 1), P.status))
          break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * kTmemCols);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = (int)(it % G::NST);
          if (!mbar_wait(&full[s], (uint32_t)((it / G::NST) & 1), P.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = saddr(smem + (size_t)s * G::STAGE);
          const uint32_t b = a + kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // A: K-major, 128-byte rows, 8-row atoms 1024 B apart; +32 B per K=16.
            // B: MN-major, 64-column atoms 8 KB apart (LBO), 8-row K groups
            //    1024 B apart (SBO); +2048 B per K=16.
            // (e4m3: K = 32 per MMA, 32 bytes as well; B K-major like A)
            const uint64_t ad = smem_desc(a + 32 * k, 16, 1024);
            const uint64_t bd = F8 ? smem_desc(b + 32 * k, 16, 1024)
                                   : smem_desc(b + 2048 * k, kBK * 64 * 2, 1024);
            mma_bf16<CG, F8>(d, ad, bd, G::IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          // the stage is free (in both CTAs) once these MMAs have read it
          mma_commit_to<CG>(saddr(&empty[s]));
          if constexpr (CG == 2) mma_commit_to<CG>(map_rank(saddr(&empty[s]), 1));
        }
        mma_commit_to<CG>(saddr(&acc_full[buf]));  // accumulator j complete
        if constexpr (CG == 2) mma_commit_to<CG>(map_rank(saddr(&acc_full[buf]), 1));
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 (this CTA's rows)
    const int q = warp & 3;
    const float alpha = F8 ? (*P.scale_a) * (*P.scale_b) : 1.f;  // FP8: sa * sb
    const uint32_t acc_empty_leader = map_rank(saddr(acc_empty), 0);
    int j = 0;
    for (int64_t t = cid; t < ntiles; t += ncl, ++j) {
      int64_t mb, nb;
      tile_coords(t, mt, nt, mb, nb);
      const int64_t row0 = mb * G::BM + rank * kBM + 32 * q;  // first row of this warp
      const int64_t m = row0 + lane, n0 = nb * kBN;
      // this row's mask words for the tile's 256 columns, fetched before the wait
      uint64_t keep[kBN / 64];
#pragma unroll
      for (int i = 0; i < kBN / 64; ++i) {
        keep[i] = RELU2 ? 0ull : ~0ull;
        if constexpr (MASK) {
          // ReLU^2 counts values, so every row of an existing tile is read
          // (rows past M have clear bits there)
          const bool in = RELU2 ? (m >> 6) < P.mask_grid_m : m < P.M;
          if (in && n0 + 64 * i < P.N)
            keep[i] = *reinterpret_cast<const uint64_t *>(
                P.mask + ((m >> 6) * P.mask_grid_n + (n0 >> 6) + i) * kTileBytes + (m & 63) * 8);
        }
      }
      // ReLU^2: this warp's 32 rows of each of the tile's four 64 x 64 tiles
      // of h hold one contiguous run of the value stream; its bounds depend
      // only on the bitmask, so they are found -- and the first two runs'
      // copies into shared memory started -- before the accumulator is ready
      uint32_t rexcl[kBN / 64], rfirst[kBN / 64];
      int64_t ra0[kBN / 64];
      int rnv[kBN / 64];
      uint8_t *vs0 = vstage + (size_t)q * kValBufs * kValStage;
      if constexpr (RELU2) {
#pragma unroll
        for (int c = 0; c < kBN / 64; ++c) {
          rexcl[c] = 0; rfirst[c] = 0; ra0[c] = 0; rnv[c] = 0;
          const int64_t tile = (row0 >> 6) * P.mask_grid_n + (n0 >> 6) + c;
          if ((row0 >> 6) < P.mask_grid_m && n0 + 64 * c < P.N) {  // warp-uniform
            const uint32_t cnt = (uint32_t)__popcll(keep[c]);
            uint32_t before = 0;
            if (row0 & 32) {  // rows 0..31 of the tile belong to the other warp
              const uint64_t ow =
                  *reinterpret_cast<const uint64_t *>(P.mask + tile * kTileBytes + lane * 8);
              before = __reduce_add_sync(0xFFFFFFFFu, (uint32_t)__popcll(ow));
            }
            uint32_t inc = cnt;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
              const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, d);
              if (lane >= d) inc += t;
            }
            const uint32_t total = __shfl_sync(0xFFFFFFFFu, inc, 31);
            const int64_t seg0 = (int64_t)P.prefix[tile] + *P.vals_offset + before;
            const int64_t a0 = (seg0 * VB) & ~(int64_t)15;
            const int64_t a1 = ((seg0 + (int64_t)total) * VB + 15) & ~(int64_t)15;
            rexcl[c] = inc - cnt;
            rfirst[c] = (uint32_t)((seg0 * VB - a0) / VB);
            ra0[c] = a0;
            rnv[c] = (int)((a1 - a0) >> 4);
          }
        }
        __syncwarp();  // the previous tile's reads of both buffers are done
#pragma unroll
        for (int c = 0; c < kValBufs; ++c) {
          const uint8_t *src = reinterpret_cast<const uint8_t *>(P.vals) + ra0[c];
          for (int v = lane; v < rnv[c]; v += 32)
            cp_async16(vs0 + (size_t)c * kValStage + v * 16, src + v * 16);
          cp_async_commit();
        }
      }
      const int buf = j & 1;
      const bool ok = mbar_wait(&acc_full[buf], (uint32_t)((j >> 1) & 1), P.status);
      tc_fence_after();
      const uint32_t zero_guard = ok ? 0xFFFFFFFFu : 0u;  // a failed wait writes zeros
      const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * kTmemCols);
#pragma unroll
      for (int c = 0; c < kBN / 64; ++c) {
        uint32_t r[64];
        tmem_ld32_nowait(tbase + (uint32_t)(64 * c), r);
        tmem_ld32_nowait(tbase + (uint32_t)(64 * c + 32), r + 32);
        tmem_wait_ld();
        const uint64_t kw = keep[c];
        uint32_t w[32];
        if constexpr (RELU2) {
          // grad_z = bit ? bf16(float(bf16(acc)) * (2k r)) : 0, r the stored
          // value at the element's rank, read from the staged run; FP8: acc
          // is scaled by sa * sb before the rounding (the GEMM's output), r
          // is the e4m3 value, and the result is multiplied by the stored
          // tensor's scale with a second rounding (grad.mul_(scale))
          if (c + 1 < kBN / 64) cp_async_wait<1>();  // this chunk's copies are in
          else cp_async_wait<0>();
          __syncwarp();
          uint8_t *vs = vs0 + (size_t)(c % kValBufs) * kValStage;
          const uint32_t first = rfirst[c], excl = rexcl[c];
          const uint16_t *sv = reinterpret_cast<const uint16_t *>(vs);
          const uint8_t *sv8 = vs;
          // grad.mul_(scale) multiplies a bf16 tensor by the 0-dim fp32 scale,
          // which torch first casts to the tensor's dtype: bf16(scale)
          const float hs = (EPI == kEpiFp8Relu2 && P.hscale)
                               ? __uint_as_float(bf16x2_rn(__float_as_uint(*P.hscale), 0u) << 16)
                               : 1.f;
          uint32_t rk = first + excl;
          // k = 1 (the reference's RELU2_SCALE): 2r is exact in bf16 and the
          // fp32 product of two bf16 values is exact, so bf16(g * 2r) is one
          // bf16x2 multiply (round to nearest even); other k: fp32 as written
          const bool two = P.two_k == 2.0f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const uint32_t g2 =  // grad_h, rounded
                F8 ? bf16x2_rn(__float_as_uint(__uint_as_float(r[2 * i]) * alpha),
                               __float_as_uint(__uint_as_float(r[2 * i + 1]) * alpha))
                   : bf16x2_rn(r[2 * i], r[2 * i + 1]);
            const uint32_t b0 = (uint32_t)(kw >> (2 * i)) & 1u;
            const uint32_t b1 = (uint32_t)(kw >> (2 * i + 1)) & 1u;
            const uint32_t u0 = VB == 1 ? code_bf16[sv8[rk]] : sv[rk];
            rk += b0;
            const uint32_t u1 = VB == 1 ? code_bf16[sv8[rk]] : sv[rk];
            rk += b1;
            uint32_t y;
            if (two) {
              y = bf16x2_mul(g2, bf16x2_mul(u0 | (u1 << 16), 0x40004000u));  // g * (2 r)
            } else {
              const float y0 = __uint_as_float(g2 << 16) * (P.two_k * __uint_as_float(u0 << 16));
              const float y1 =
                  __uint_as_float(g2 & 0xFFFF0000u) * (P.two_k * __uint_as_float(u1 << 16));
              y = bf16x2_rn(__float_as_uint(y0), __float_as_uint(y1));
            }
            if constexpr (EPI == kEpiFp8Relu2) {
              if (P.hscale)
                y = bf16x2_rn(__float_as_uint(__uint_as_float(y << 16) * hs),
                              __float_as_uint(__uint_as_float(y & 0xFFFF0000u) * hs));
            }
            const uint32_t keep_w = (b0 ? 0x0000FFFFu : 0u) | (b1 ? 0xFFFF0000u : 0u);
            w[i] = y & keep_w & zero_guard;
          }
          if (c + kValBufs < kBN / 64) {  // refill this buffer with chunk c + 2
            __syncwarp();
            const uint8_t *src = reinterpret_cast<const uint8_t *>(P.vals) + ra0[c + kValBufs];
            for (int v = lane; v < rnv[c + kValBufs]; v += 32)
              cp_async16(vs + v * 16, src + v * 16);
          }
          cp_async_commit();  // (possibly empty) group: the wait counts stay uniform
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            // mask bits 2i, 2i+1 -> 0x0000FFFF / 0xFFFF0000 halves
            const uint32_t two = (uint32_t)(kw >> (2 * i)) & 3u;
            const uint32_t keep_w = ((two & 1u) ? 0x0000FFFFu : 0u) | ((two & 2u) ? 0xFFFF0000u : 0u);
            if constexpr (F8)
              w[i] = bf16x2_rn(__float_as_uint(__uint_as_float(r[2 * i]) * alpha),
                               __float_as_uint(__uint_as_float(r[2 * i + 1]) * alpha)) &
                     zero_guard;
            else
              w[i] = bf16x2_rn(r[2 * i], r[2 * i + 1]) & keep_w & zero_guard;
          }
        }
        const int64_t n = n0 + 64 * c;
        if (P.c_tma) {
          // stage row `lane` of this warp's 32 x 64 box: 16-byte chunk i at
          // chunk i ^ (row & 7) (the 128-byte swizzle of the store's tensor
          // map; conflict-free), then one lane stores the box with TMA
          uint8_t *box = epi + (size_t)(q * 2 + (c & 1)) * kEpiBox;
          if (lane == 0)  // the store that last read this box is done reading
            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<uint4 *>(box + lane * 128 + ((i ^ (lane & 7)) * 16)) =
                make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0 && n < P.N && row0 < P.M) {
            asm volatile(
                "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                    reinterpret_cast<uint64_t>(&tmC)),
                "r"((int)n), "r"((int)row0), "r"(saddr(box))
                : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
        } else if (m < P.M) {
          for (int i = 0; i < 64 && n + i < P.N; ++i)
            reinterpret_cast<uint16_t *>(P.C + (m * P.ldc + n) * 2)[i] =
                (uint16_t)(w[i >> 1] >> (16 * (i & 1)));
        }
      }
      // this warp is done with accumulator buf (the leader's barrier counts
      // the epilogue warps of both CTAs)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + (uint32_t)(8 * buf));
    }
  }
  if (warp >= 2 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync();  // no CTA leaves while its peer may signal it
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(2 * kTmemCols)
                   : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                   "r"(2 * kTmemCols)
                   : "memory");
  }
}

// ---------------------------------------------------------------------------
// K5 -- the weight-gradient GEMM with the reconstruct fused into its B
// producer (AspB / AspRelu2B, lib_sparse/src/sparse_matmul.py:9-47, :91-132):
//
//   C[D, H] = g^T[D, T] . h[T, H]      h = unpack(stored)  or  k * unpack(stored)^2
//
// g is row-major [T, D] (grad_output), so A = g^T is MN-major; h is a bf16
// bitsparse tensor [T, H].  A 64-token x 64-column box of h is exactly one
// compressed tile, expanded by producer warps straight into the 128-byte
// swizzled MN-major layout tcgen05.mma reads: the dense h never exists in
// HBM.  Expansion runs on the CUDA cores, so each expanded tile is made to
// feed as much tensor-core work as TMEM holds: a CTA pair (cta_group::2) owns
// an (NMB x 256) x 128 block of C -- NMB m-blocks of 256 rows, one TMEM
// accumulator of 128 columns each -- and per 64-token K step expands ONE
// tile per CTA (its 64 of the 128 columns) for NMB MMAs of 256 x 128 x 64.
// Small outputs split K over KS pair tiles (fp32 partials, summed in order
// by `dw_reduce_kernel`) so that every SM pair has work.
//   warp 0      producer: the NMB m-blocks' A boxes by TMA (two 64 x 64 atoms
//               each); the tile's bitmask and value run (one 16-byte aligned
//               superset) by 1-D bulk copies into a compressed-data slot, the
//               tile prefixes read ahead through a cp.async ring;
//   warp 1      MMA issuer (leader CTA);
//   warps 2..5  epilogue: TMEM -> bf16 -> TMA store, or fp32 partials;
//   warps 6..13 expanders: warp 6 + e expands rows 8e .. 8e + 7 of the tile
//               -- lane = (row, 8-column chunk): the chunk's mask byte, its
//               first rank from a scan of the row counts, the ranks of its 8
//               positions from one nibble-packed prefix sum, the set values
//               read from the staged run, one 16-byte swizzled store -- then
//               fence.proxy.async and the stage arrival (below).
// Stage completion: the leader's TMA bytes and its expanders' local arrivals
// land on the leader's barrier; each of the peer's expander warps completes 4
// transaction bytes on it with st.async (asynchronous, released at cluster
// scope) -- a blocking cluster-scope arrive costs 0.6-1 us per warp.
// All waits are bounded (BS_STATUS_TIMEOUT); copies in flight are waited for
// before the CTA exits; TMEM is always freed.
constexpr int kThreadsD = 448;  // 14 warps
constexpr int kDwBN = 128;      // columns of C per pair tile (64 per CTA: one tile of h)
constexpr int kDwEpiBytes = 4 * kEpiBox;  // one staging box per epilogue warp
template <int NMB>
struct DwCfg {
  static constexpr int BM = 2 * kBM;              // rows of one m-block (pair)
  static constexpr int MG = NMB * BM;             // rows of C per pair tile
  static constexpr int ABYTES = NMB * 2 * 8192;   // this CTA's 128 rows of each m-block
  static constexpr int BBYTES = 8192;             // this CTA's 64 columns: one tile
  static constexpr int STAGE = ABYTES + BBYTES;
  static constexpr int RS = 3;                    // compressed-data slots
  static constexpr int RMETA = 16, RMASK = kTileBytes, RVALS = 8192 + 32;
  static constexpr int RSLOT = RMETA + RMASK + RVALS;
  static constexpr int LA = 8;                    // prefix read-ahead (steps)
  static constexpr int NAB = NMB <= 2 ? 2 : 1;    // accumulator sets in TMEM (512 columns)
  static constexpr size_t FIXED = 1024 + kDwEpiBytes + (size_t)RS * RSLOT + LA * 16 + 512;
  static constexpr int NSTF = (int)((227 * 1024 - FIXED) / STAGE);
  static constexpr int NST = NSTF > 6 ? 6 : NSTF;
  static constexpr size_t SMEM = FIXED + (size_t)NST * STAGE;
  // fp32 accumulator, bf16 A and B, both MN-major, N = 128, M = 256
  static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) |
                                    (1u << 16) | ((uint32_t)(kDwBN >> 3) << 17) |
                                    ((uint32_t)(BM >> 4) << 24);
  static_assert(RSLOT % 16 == 0, "bulk-copy destinations stay 16-byte aligned");
  static_assert(STAGE % 1024 == 0 && kDwEpiBytes % 1024 == 0,
                "stages and staging boxes stay on 1024-byte boundaries");
  static_assert(NST >= 2, "a pipeline needs two stages");
  static_assert(NAB * NMB * kDwBN <= 512, "accumulators fit TMEM");
};

struct DwParams {
  uint8_t *C;
  int64_t M, N, K, ldc;      // D, H, T
  float *part;               // split K: fp32 partials [ks][M][N], else null
  int ks, kspan;             // K splits, 64-token blocks per split
  int64_t mt, nt;            // pair tiles along M (m-groups) and N
  const uint8_t *vals;       // stored values (bf16), 16-byte aligned base
  const uint8_t *bitmask;    // [grid_m * grid_n] tiles of 512 bytes
  const uint32_t *prefix;    // [grid_m * grid_n + 1]
  const int64_t *vals_offset;
  int64_t grid_n;            // tile columns of h: ceil(H / 64)
  int c_tma;
  int32_t *status;
};

__device__ __forceinline__ void mbar_arrive_local(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
// Bounded wait with cluster-scope acquire (the barrier counts an arrival
// released by the peer CTA of the pair).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity,
                                                  int32_t *status) {
  for (uint32_t n = 0; n < kMaxPolls; ++n) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  status_or(status, BS_STATUS_TIMEOUT);
  return false;
}
// Explicit shared-space accesses (the aligned dynamic shared-memory base is
// formed through an integer, which hides the state space from the compiler).
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint64_t lds_u64(uint32_t a) {
  uint64_t v;
  asm volatile("ld.shared.u64 %0, [%1];" : "=l"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(saddr(dst)), "l"(src) : "memory");
}

// Pair tile t -> (K split, m-group, n-block): n fastest, so the pairs working
// at the same time share their A rows (and K range) in L2.
__device__ __forceinline__ void dw_tile(const DwParams &P, int64_t t, int &split, int64_t &mg,
                                        int64_t &nb, int &kb0, int &kb1, int nk) {
  nb = t % P.nt;
  const int64_t r = t / P.nt;
  mg = r % P.mt;
  split = (int)(r / P.mt);
  kb0 = split * P.kspan;
  kb1 = kb0 + P.kspan < nk ? kb0 + P.kspan : nk;
}

template <int NMB, bool RELU2>
__global__ void __launch_bounds__(kThreadsD, 1)
    dw_unpack_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmC, const DwParams P) {
  using G = DwCfg<NMB>;
  constexpr int CG = 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // stages and the epilogue's swizzled staging boxes on 1024-byte
  // boundaries (the 128-byte swizzle atoms), then the compressed-data slots
  uint8_t *epi = smem + (size_t)G::NST * G::STAGE;
  uint8_t *raw = epi + kDwEpiBytes;
  uint32_t *pref = reinterpret_cast<uint32_t *>(raw + (size_t)G::RS * G::RSLOT);  // [LA][4]
  uint64_t *full = reinterpret_cast<uint64_t *>(pref + 4 * G::LA);
  uint64_t *empty = full + G::NST;
  uint64_t *rfull = empty + G::NST;
  uint64_t *rempty = rfull + G::RS;
  uint64_t *acc_full = rempty + G::RS;
  uint64_t *acc_empty = acc_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
  uint32_t *sig = tmem_slot + 4;  // [8] the peer expanders' st.async targets (values unused)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t cid = (int64_t)blockIdx.x / CG, ncl = (int64_t)gridDim.x / CG;
  const int nk = (int)((P.K + kBK - 1) / kBK);
  const int64_t ntiles = P.mt * P.nt * P.ks;

  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    for (int s = 0; s < G::NST; ++s) {
      // leader: its A arrival + its 8 expander warps (the peer's expanders
      // complete transaction bytes on it with st.async)
      mbar_init(&full[s], 1 + 8);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < G::RS; ++r) {
      mbar_init(&rfull[r], 1);
      mbar_init(&rempty[r], 8);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4 * CG);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // this CTA pair's steps: the K blocks of its tiles cid, cid + ncl, ...
  int64_t nsteps = 0;
  for (int64_t t = cid; t < ntiles; t += ncl) {
    int split, kb0, kb1;
    int64_t mg, nb;
    dw_tile(P, t, split, mg, nb, kb0, kb1, nk);
    nsteps += kb1 > kb0 ? kb1 - kb0 : 0;
  }

  if (warp == 0) {
    if (lane == 0) {
      const int64_t voff = *P.vals_offset;
      // step cursor: tile t, its K range, its tile column of h and whether
      // that tile exists (0 past the right edge of h)
      struct Cursor {
        int64_t t, mg, nb, c0;
        int kb, kb1, ntl;
      };
      auto at_tile = [&](Cursor &c, int64_t t) {
        for (;; t += ncl) {
          c.t = t;
          if (t >= ntiles) return;
          int split;
          dw_tile(P, t, split, c.mg, c.nb, c.kb, c.kb1, nk);
          c.c0 = c.nb * 2 + (int64_t)rank;
          c.ntl = c.c0 < P.grid_n ? 1 : 0;
          if (c.kb < c.kb1) return;  // (an empty split has no steps)
        }
      };
      auto advance = [&](Cursor &c) {
        if (++c.kb == c.kb1) at_tile(c, c.t + ncl);
      };
      Cursor ahead;
      at_tile(ahead, cid);
      int ring_in = 0;
      auto issue_prefix = [&]() {
        if (ahead.t < ntiles) {
          const int64_t tf = (int64_t)ahead.kb * P.grid_n + ahead.c0;
          uint32_t *e = pref + 4 * ring_in;
          if (ahead.ntl) {
            cp_async4(e, P.prefix + tf);
            cp_async4(e + 1, P.prefix + tf + 1);
          }
          advance(ahead);
        }
        cp_async_commit();  // (possibly empty) group: one per step
        if (++ring_in == G::LA) ring_in = 0;
      };
      for (int i = 0; i < G::LA; ++i) issue_prefix();
      Cursor cur;
      at_tile(cur, cid);
      int s = 0, rs = 0, ring = 0;
      uint32_t sph = 0, rph = 0;
      bool ok = true;
      int64_t j = 0;
      for (; j < nsteps && ok; ++j) {
        if (j >= G::NST && !mbar_wait(&empty[s], sph ^ 1u, P.status)) {
          ok = false;
          break;
        }
        uint8_t *a = smem + (size_t)s * G::STAGE;
        if (leader) mbar_expect_tx(&full[s], 2 * G::ABYTES + 8 * 4);
        const uint32_t bar = map_rank(saddr(&full[s]), 0);
#pragma unroll
        for (int mi = 0; mi < NMB; ++mi) {
          const int ax = (int)(cur.mg * G::MG + mi * G::BM + rank * kBM);
          tma_load_2d_pair(a + mi * 16384, &tmA, ax, cur.kb * kBK, bar);
          tma_load_2d_pair(a + mi * 16384 + 8192, &tmA, ax + 64, cur.kb * kBK, bar);
        }
        if (j >= G::RS && !mbar_wait(&rempty[rs], rph ^ 1u, P.status)) {
          ok = false;
          break;
        }
        const int ntl = cur.ntl;
        const int64_t tfirst = (int64_t)cur.kb * P.grid_n + cur.c0;
        cp_async_wait<G::LA - 1>();  // step j's prefixes are in
        const uint32_t *e = pref + 4 * ring;
        uint8_t *slot = raw + (size_t)rs * G::RSLOT;
        uint32_t mbytes = 0, vbytes = 0;
        int64_t a0 = 0;
        uint32_t *meta = reinterpret_cast<uint32_t *>(slot);
        if (ntl) {
          const uint32_t p0 = e[0], p1 = e[1];
          const int64_t b0 = (voff + p0) * 2, b1 = (voff + p1) * 2;
          a0 = b0 & ~(int64_t)15;
          const int64_t a1 = (b1 + 15) & ~(int64_t)15;
          vbytes = p1 > p0 ? (uint32_t)(a1 - a0) : 0u;  // no values: no copy
          mbytes = kTileBytes;
          meta[0] = (uint32_t)((b0 - a0) >> 1);  // first value's position in the slot
        }
        meta[2] = (uint32_t)ntl;
        issue_prefix();  // the ring entry just read is reused for step j + LA
        mbar_expect_tx(&rfull[rs], mbytes + vbytes);  // also releases the meta words
        if (mbytes) bulk_load(slot + G::RMETA, P.bitmask + tfirst * kTileBytes, mbytes, &rfull[rs]);
        if (vbytes) bulk_load(slot + G::RMETA + G::RMASK, P.vals + a0, vbytes, &rfull[rs]);
        advance(cur);
        if (++ring == G::LA) ring = 0;
        if (++s == G::NST) { s = 0; sph ^= 1u; }
        if (++rs == G::RS) { rs = 0; rph ^= 1u; }
      }
      cp_async_wait<0>();
      // every copy landed before the CTA may exit
      for (int64_t i = j - G::RS < 0 ? 0 : j - G::RS; i < j; ++i)
        mbar_wait(&rfull[i % G::RS], (uint32_t)((i / G::RS) & 1), P.status);
      if (leader)
        for (int64_t i = j - G::NST < 0 ? 0 : j - G::NST; i < j; ++i)
          mbar_wait_cluster(&full[i % G::NST], (uint32_t)((i / G::NST) & 1), P.status);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int64_t it = 0;
      int jt = 0;
      bool ok = true;
      for (int64_t t = cid; t < ntiles && ok; t += ncl) {
        int split, kb0, kb1;
        int64_t mg, nb;
        dw_tile(P, t, split, mg, nb, kb0, kb1, nk);
        if (kb1 <= kb0) continue;  // the epilogue skips it too
        const int buf = jt % G::NAB;
        const int use = jt / G::NAB;
        if (use >= 1 && !mbar_wait(&acc_empty[buf], (uint32_t)((use - 1) & 1), P.status)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(buf * NMB * kDwBN);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = (int)(it % G::NST);
          if (!mbar_wait_cluster(&full[s], (uint32_t)((it / G::NST) & 1), P.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = saddr(smem + (size_t)s * G::STAGE);
          const uint32_t b = a + G::ABYTES;
#pragma unroll
          for (int mi = 0; mi < NMB; ++mi) {
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              // both MN-major: 64-element atoms 8 KB apart (LBO), 8-row K
              // groups 1024 B apart (SBO); +2048 B per K = 16
              const uint64_t ad = smem_desc(a + mi * 16384 + 2048 * k, 8192, 1024);
              const uint64_t bd = smem_desc(b + 2048 * k, 8192, 1024);
              mma_bf16<CG>(d0 + (uint32_t)(mi * kDwBN), ad, bd, G::IDESC,
                           (kb > kb0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit_to<CG>(saddr(&empty[s]));
          mma_commit_to<CG>(map_rank(saddr(&empty[s]), 1));
        }
        mma_commit_to<CG>(saddr(&acc_full[buf]));
        mma_commit_to<CG>(map_rank(saddr(&acc_full[buf]), 1));
        ++jt;
      }
    }
  } else if (warp < 6) {
    // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 (this CTA's rows)
    const int q = warp & 3;
    const uint32_t acc_empty_leader = map_rank(saddr(acc_empty), 0);
    uint8_t *box = epi + (size_t)q * kEpiBox;
    int jt = 0;
    for (int64_t t = cid; t < ntiles; t += ncl) {
      int split, kb0, kb1;
      int64_t mg, nb;
      dw_tile(P, t, split, mg, nb, kb0, kb1, nk);
      if (kb1 <= kb0) continue;
      const int buf = jt % G::NAB;
      const bool ok = mbar_wait(&acc_full[buf], (uint32_t)((jt / G::NAB) & 1), P.status);
      tc_fence_after();
      const uint32_t zero_guard = ok ? 0xFFFFFFFFu : 0u;
#pragma unroll 1
      for (int mi = 0; mi < NMB; ++mi) {
        const int64_t row0 = mg * G::MG + mi * G::BM + rank * kBM + 32 * q;
        const int64_t m = row0 + lane;
        const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) +
                               (uint32_t)((buf * NMB + mi) * kDwBN);
#pragma unroll 1
        for (int c = 0; c < kDwBN / 64; ++c) {
          const int64_t n = nb * kDwBN + 64 * c;
          uint32_t r[64];
          tmem_ld32_nowait(tbase + (uint32_t)(64 * c), r);
          tmem_ld32_nowait(tbase + (uint32_t)(64 * c + 32), r + 32);
          tmem_wait_ld();
          if (row0 >= P.M || n >= P.N) continue;  // (warp-uniform)
          if (P.part) {  // split K: this split's fp32 partial row
            if (m < P.M) {
              float *dst = P.part + ((int64_t)split * P.M + m) * P.N + n;
              if (n + 64 <= P.N && (P.N & 3) == 0) {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                  *reinterpret_cast<uint4 *>(dst + 4 * i) =
                      make_uint4(r[4 * i] & zero_guard, r[4 * i + 1] & zero_guard,
                                 r[4 * i + 2] & zero_guard, r[4 * i + 3] & zero_guard);
              } else {
                for (int i = 0; i < 64 && n + i < P.N; ++i)
                  dst[i] = __uint_as_float(r[i] & zero_guard);
              }
            }
            continue;
          }
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = bf16x2_rn(r[2 * i], r[2 * i + 1]) & zero_guard;
          if (P.c_tma) {
            if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i)
              *reinterpret_cast<uint4 *>(box + lane * 128 + ((i ^ (lane & 7)) * 16)) =
                  make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              asm volatile(
                  "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                      reinterpret_cast<uint64_t>(&tmC)),
                  "r"((int)n), "r"((int)row0), "r"(saddr(box))
                  : "memory");
              asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
          } else if (m < P.M) {
            for (int i = 0; i < 64 && n + i < P.N; ++i)
              reinterpret_cast<uint16_t *>(P.C + (m * P.ldc + n) * 2)[i] =
                  (uint16_t)(w[i >> 1] >> (16 * (i & 1)));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + (uint32_t)(8 * buf));
      ++jt;
    }
  } else {
    // expanders: warp 6 + e -> rows 8e .. 8e + 7 of this CTA's tile
    const int e = warp - 6;
    const int r0 = 8 * e;
    const uint32_t full_leader = map_rank(saddr(full), 0);
    const uint32_t sig_leader = map_rank(saddr(sig), 0);
    int s = 0, rs = 0;
    uint32_t sph = 0, rph = 0;
    for (int64_t j = 0; j < nsteps; ++j) {
      if (!mbar_wait(&rfull[rs], rph, P.status)) break;
      if (j >= G::NST && !mbar_wait(&empty[s], sph ^ 1u, P.status)) break;
      const uint32_t slot = saddr(raw + (size_t)rs * G::RSLOT);
      const uint32_t box = saddr(smem + (size_t)s * G::STAGE + G::ABYTES);
      if (lds_u32(slot + 8)) {
        const uint32_t mw = slot + G::RMETA;           // the tile's 64 row words
        const uint32_t sv = slot + G::RMETA + G::RMASK;  // staged values (bf16)
        // values of the tile's rows before this warp's 8
        uint32_t before = 0;
        if (e) {
          const uint64_t wa = lds_u64(mw + 8 * lane), wb = lds_u64(mw + 8 * (32 + lane));
          before = (lane < r0 ? (uint32_t)__popcll(wa) : 0u) +
                   (lane + 32 < r0 ? (uint32_t)__popcll(wb) : 0u);
          before = __reduce_add_sync(0xFFFFFFFFu, before);
        }
        // lanes l, l + 8, l + 16, l + 24 hold row r0 + l: its word and the
        // slot position of its first value
        const uint64_t my = lds_u64(mw + 8 * (r0 + (lane & 7)));
        const uint32_t cnt = (uint32_t)__popcll(my);
        uint32_t inc = cnt;
#pragma unroll
        for (int d = 1; d < 8; d <<= 1) {
          const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, inc, d, 8);
          if ((lane & 7) >= d) inc += v;
        }
        const uint32_t rowbase = lds_u32(slot) + before + inc - cnt;
        const uint32_t mlo = (uint32_t)my, mhi = (uint32_t)(my >> 32);
        const int c = lane & 7;
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const int rl = 4 * st + (lane >> 3);  // row within this warp's 8
          const uint32_t wlo = __shfl_sync(0xFFFFFFFFu, mlo, rl);
          const uint32_t whi = __shfl_sync(0xFFFFFFFFu, mhi, rl);
          uint32_t p = __shfl_sync(0xFFFFFFFFu, rowbase, rl);
          const uint64_t wr = ((uint64_t)whi << 32) | wlo;
          const uint32_t mbyte = (uint32_t)(wr >> (8 * c)) & 0xFFu;
          p += (uint32_t)__popcll(wr & ((1ull << (8 * c)) - 1ull));
          uint32_t o[4] = {0, 0, 0, 0};
          if (mbyte) {
            // bit i -> nibble i, then nibble i of x * 0x11111111 - x = set
            // bits below position i (at most 7: no carries between nibbles)
            uint32_t x = (mbyte | (mbyte << 12)) & 0x000F000Fu;
            x = (x | (x << 6)) & 0x03030303u;
            x = (x | (x << 3)) & 0x11111111u;
            const uint32_t rk = x * 0x11111111u - x;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint32_t v =
                  ((mbyte >> i) & 1u) ? lds_u16(sv + 2 * (p + ((rk >> (4 * i)) & 0xFu))) : 0u;
              o[i >> 1] |= v << (16 * (i & 1));
            }
            if constexpr (RELU2) {  // k * v * v with k = 1: one bf16 product
#pragma unroll
              for (int i = 0; i < 4; ++i) o[i] = bf16x2_mul(o[i], o[i]);
            }
          }
          const int row = r0 + rl;
          sts_v4(box + row * 128 + ((c ^ (row & 7)) * 16), o[0], o[1], o[2], o[3]);
        }
      } else {  // no tile here (right edge of h): zero columns
#pragma unroll
        for (int i = 0; i < 2; ++i) sts_v4(box + r0 * 128 + (i * 32 + lane) * 16, 0, 0, 0, 0);
      }
      fence_proxy_async_smem();  // B writes (and slot reads) before the async proxy's use
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_local(&rempty[rs]);
        if (leader) {
          mbar_arrive_local(&full[s]);
        } else {
          // 4 bytes into the leader's signal word with a complete-tx on its
          // stage barrier: asynchronous, released at cluster scope, so this
          // warp does not wait for the cluster-wide visibility of its tile
          asm volatile(
              "st.async.shared::cluster.mbarrier::complete_tx::bytes.u32 [%0], %1, [%2];" ::"r"(
                  sig_leader + (uint32_t)(4 * e)),
              "r"((uint32_t)j), "r"(full_leader + (uint32_t)(8 * s))
              : "memory");
        }
      }
      if (++s == G::NST) { s = 0; sph ^= 1u; }
      if (++rs == G::RS) { rs = 0; rph ^= 1u; }
    }
  }
  if (warp >= 2 && warp < 6 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
}

// Split K: C = bf16(sum over the splits, in order, of the fp32 partials).
__global__ void __launch_bounds__(256) dw_reduce_kernel(const float *part, int ks, int64_t M,
                                                         int64_t N, uint8_t *C, int64_t ldc) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc = part[i];
    for (int k = 1; k < ks; ++k) acc += part[(int64_t)k * total + i];
    const int64_t m = i / N, n = i - m * N;
    reinterpret_cast<uint16_t *>(C + (m * ldc + n) * 2)[0] =
        (uint16_t)bf16x2_rn(__float_as_uint(acc), 0u);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
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

// 2-D bf16 (or, with eb = 1, 8-bit) tensor map: rows x cols (cols
// contiguous), box box_cols x box_rows, 128-byte swizzle.
bool make_map(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int64_t ld,
              uint32_t box_cols, uint32_t box_rows, int eb = 2) {
  EncodeTiledFn encode = encode_tiled();
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * eb};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, eb == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                2, const_cast<void *>(base), dims,
                strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI, int CG>
int launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tc,
                const GemmParams &P, cudaStream_t st) {
  using G = GemmCfg<CG, EPI>;
  static_assert(G::SMEM <= 227 * 1024, "shared memory of one CTA");
  auto kernel = gemm_mask_kernel<EPI, CG>;
  // The shared-memory attribute is per device and the SM count may differ
  // between devices: both are set up once for each device this process uses.
  constexpr int kMaxDev = 64;
  static std::mutex mu;
  static int sms_of[kMaxDev] = {};  // 0: not yet set up on that device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return BS_ERR_LAUNCH;
  int sms;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!sms_of[dev]) {
      int n = 0;
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)G::SMEM) != cudaSuccess ||
          cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return BS_ERR_LAUNCH;
      sms_of[dev] = n;
    }
    sms = sms_of[dev];
  }
  const int64_t tiles = ((P.M + G::BM - 1) / G::BM) * ((P.N + kBN - 1) / kBN);
  const int64_t slots = sms / CG;  // persistent: one CTA (pair) per SM (pair)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(CG * (tiles < slots ? tiles : slots)));
  cfg.blockDim = dim3(kThreadsG);
  cfg.dynamicSmemBytes = G::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, P) != cudaSuccess) return BS_ERR_LAUNCH;
  return BS_OK;
}

}  // namespace
}  // namespace bs

using namespace bs;

namespace bs {
namespace {
// Shared by the entry points: checks, tensor maps, and the launch of the
// epilogue variant EPI (P's epilogue fields already set by the caller).
int gemm_run(const void *A, int64_t lda, const void *B, int64_t ldb, void *C, int64_t ldc,
             int64_t M, int64_t N, int64_t K, int epi, GemmParams &P, cudaStream_t st) {
  if (M < 0 || N < 0 || K < 0) return BS_ERR_SHAPE;
  if (M == 0 || N == 0) return BS_OK;
  if (!A || !B || !C) return BS_ERR_ARG;
  if (lda < K || (epi != kEpiFp8 && epi != kEpiFp8Relu2 && ldb < N) || ldc < N)
    return BS_ERR_SHAPE;
  if (M >= ((int64_t)1 << 31) || N >= ((int64_t)1 << 31) || K >= ((int64_t)1 << 31))
    return BS_ERR_TOO_LARGE;
  // TMA: 16-byte aligned bases and row strides (FP8: B is B^T [N, K], ldb >= K)
  const bool f8 = epi == kEpiFp8 || epi == kEpiFp8Relu2;
  const int eb = f8 ? 1 : 2;
  if (f8 && ldb < K) return BS_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15) ||
      ((lda * eb) & 15) || ((ldb * eb) & 15))
    return BS_ERR_ALIGN;
  if (P.mask && (reinterpret_cast<uintptr_t>(P.mask) & 7)) return BS_ERR_ALIGN;
  P.C = static_cast<uint8_t *>(C);
  P.M = M; P.N = N; P.K = K; P.ldc = ldc;
  P.mask_grid_n = (N + kTileN - 1) / kTileN;
  P.mask_grid_m = (M + kTileM - 1) / kTileM;
  P.c_tma = ((reinterpret_cast<uintptr_t>(C) & 15) == 0) && ((ldc * 2) % 16 == 0);
  CUtensorMap ta, tb, tc;
  if (K == 0) {  // empty reduction: C = 0 (so is every epilogue of it)
    for (int64_t r = 0; r < M; ++r)
      if (cudaMemsetAsync(static_cast<uint8_t *>(C) + r * ldc * 2, 0, (size_t)N * 2, st) !=
          cudaSuccess)
        return BS_ERR_LAUNCH;
    return BS_OK;
  }
  if (f8) {
    if (!make_map(&ta, A, M, K, lda, 128, kBM, 1) || !make_map(&tb, B, N, K, ldb, 128, 64, 1))
      return BS_ERR_ALIGN;
  } else if (!make_map(&ta, A, M, K, lda, kBK, kBM) || !make_map(&tb, B, K, N, ldb, 64, kBK)) {
    return BS_ERR_ALIGN;
  }
  // CTA pairs (cta_group::2) once there are two 128-row blocks to share
  const bool pair = M >= 2 * kBM && !getenv("BS_GEMM_ONE_CTA");
  if (P.c_tma && !make_map(&tc, C, M, N, ldc, 64, 32)) P.c_tma = 0;
  if (!P.c_tma) tc = ta;  // unused
  if (pair) {
    if (epi == kEpiFp8) return launch_gemm<kEpiFp8, 2>(ta, tb, tc, P, st);
    if (epi == kEpiFp8Relu2) return launch_gemm<kEpiFp8Relu2, 2>(ta, tb, tc, P, st);
    if (epi == kEpiRelu2) return launch_gemm<kEpiRelu2, 2>(ta, tb, tc, P, st);
    return epi == kEpiMask ? launch_gemm<kEpiMask, 2>(ta, tb, tc, P, st)
                           : launch_gemm<kEpiNone, 2>(ta, tb, tc, P, st);
  }
  if (epi == kEpiFp8) return launch_gemm<kEpiFp8, 1>(ta, tb, tc, P, st);
  if (epi == kEpiFp8Relu2) return launch_gemm<kEpiFp8Relu2, 1>(ta, tb, tc, P, st);
  if (epi == kEpiRelu2) return launch_gemm<kEpiRelu2, 1>(ta, tb, tc, P, st);
  return epi == kEpiMask ? launch_gemm<kEpiMask, 1>(ta, tb, tc, P, st)
                         : launch_gemm<kEpiNone, 1>(ta, tb, tc, P, st);
}
}  // namespace
}  // namespace bs

extern "C" int bs_gemm_bf16_mask(const void *A, int64_t lda, const void *B, int64_t ldb,
                                 void *C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                                 const uint8_t *mask, int32_t *status, void *stream) {
  GemmParams P{};
  P.mask = mask;
  P.status = status;
  return gemm_run(A, lda, B, ldb, C, ldc, M, N, K, mask ? kEpiMask : kEpiNone, P,
                  static_cast<cudaStream_t>(stream));
}

extern "C" int bs_gemm_bf16_relu2(const void *A, int64_t lda, const void *B, int64_t ldb,
                                  void *C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                                  const void *vals, const uint8_t *bitmask,
                                  const uint32_t *prefix, const int64_t *vals_offset, float k,
                                  int32_t *status, void *stream) {
  if (!vals || !bitmask || !prefix || !vals_offset) return BS_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(vals) & 15) return BS_ERR_ALIGN;  // 16-byte staging loads
  GemmParams P{};
  P.mask = bitmask;
  P.vals = static_cast<const uint16_t *>(vals);
  P.prefix = prefix;
  P.vals_offset = vals_offset;
  P.two_k = 2.0f * k;
  P.status = status;
  return gemm_run(A, lda, B, ldb, C, ldc, M, N, K, kEpiRelu2, P,
                  static_cast<cudaStream_t>(stream));
}

extern "C" int bs_gemm_fp8(const void *A, int64_t lda, const void *Bt, int64_t ldb, void *C,
                           int64_t ldc, int64_t M, int64_t N, int64_t K, const float *scale_a,
                           const float *scale_b, int32_t *status, void *stream) {
  if (!scale_a || !scale_b) return BS_ERR_ARG;
  GemmParams P{};
  P.scale_a = scale_a;
  P.scale_b = scale_b;
  P.status = status;
  return gemm_run(A, lda, Bt, ldb, C, ldc, M, N, K, kEpiFp8, P,
                  static_cast<cudaStream_t>(stream));
}

extern "C" int bs_gemm_fp8_relu2(const void *A, int64_t lda, const void *Bt, int64_t ldb,
                                 void *C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                                 const float *scale_a, const float *scale_b, const void *vals,
                                 const uint8_t *bitmask, const uint32_t *prefix,
                                 const int64_t *vals_offset, float k, const float *hscale,
                                 int32_t *status, void *stream) {
  if (!scale_a || !scale_b || !vals || !bitmask || !prefix || !vals_offset) return BS_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(vals) & 15) return BS_ERR_ALIGN;  // 16-byte staging loads
  GemmParams P{};
  P.scale_a = scale_a;
  P.scale_b = scale_b;
  P.mask = bitmask;
  P.vals = static_cast<const uint16_t *>(vals);
  P.prefix = prefix;
  P.vals_offset = vals_offset;
  P.two_k = 2.0f * k;
  P.hscale = hscale;
  P.status = status;
  return gemm_run(A, lda, Bt, ldb, C, ldc, M, N, K, kEpiFp8Relu2, P,
                  static_cast<cudaStream_t>(stream));
}

namespace bs {
namespace {
// The K5 plan: NMB m-blocks per pair tile (as many as TMEM holds, spread
// evenly over the m-groups), the pair tiles, and a K split when the tiles
// alone leave SM pairs idle (at least 16 K blocks per split).
struct DwPlan {
  int nmb, ks, kspan, nk;
  int64_t mt, nt;
};
DwPlan dw_plan(int64_t T, int64_t D, int64_t H, int sms) {
  DwPlan p{};
  const int64_t mb = (D + 2 * kBM - 1) / (2 * kBM);
  // at most 4 m-blocks per pair tile (TMEM); BS_DW_MAX_NMB lowers the cap
  // for measurements (more stages fit with fewer m-blocks, at the cost of
  // expanding each tile for more m-groups: 3 and 4 measure alike, 2 slower)
  static const int max_nmb = [] {
    const char *e = getenv("BS_DW_MAX_NMB");
    const int v = e ? atoi(e) : 4;
    return v < 1 ? 1 : (v > 4 ? 4 : v);
  }();
  p.mt = (mb + max_nmb - 1) / max_nmb;
  p.nmb = (int)((mb + p.mt - 1) / p.mt);
  p.nt = (H + kDwBN - 1) / kDwBN;
  p.nk = (int)((T + kBK - 1) / kBK);
  const int64_t tiles = p.mt * p.nt, pairs = sms / 2;
  int64_t ks = 1;
  if (tiles < pairs && p.nk >= 32) {
    ks = pairs / tiles;
    if (ks > p.nk / 16) ks = p.nk / 16;
    if (ks < 1) ks = 1;
  }
  p.kspan = (int)((p.nk + ks - 1) / ks);
  p.ks = p.kspan ? (p.nk + p.kspan - 1) / p.kspan : 1;  // no empty split
  return p;
}
int dev_sms() {
  constexpr int kMaxDev = 64;
  static int sms_of[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 0;
  if (!sms_of[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    sms_of[dev] = n;  // benign race: every writer stores the same value
  }
  return sms_of[dev];
}
template <int NMB, bool RELU2>
int launch_dw(const CUtensorMap &ta, const CUtensorMap &tc, const DwParams &P, int sms,
              cudaStream_t st) {
  using G = DwCfg<NMB>;
  static_assert(G::SMEM <= 227 * 1024, "shared memory of one CTA");
  auto kernel = dw_unpack_kernel<NMB, RELU2>;
  constexpr int kMaxDev = 64;
  static std::mutex mu;
  static bool set_on[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return BS_ERR_LAUNCH;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!set_on[dev]) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)G::SMEM) != cudaSuccess)
        return BS_ERR_LAUNCH;
      set_on[dev] = true;
    }
  }
  const int64_t tiles = P.mt * P.nt * P.ks;
  const int64_t slots = sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * (tiles < slots ? tiles : slots)));
  cfg.blockDim = dim3(kThreadsD);
  cfg.dynamicSmemBytes = G::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, ta, tc, P) != cudaSuccess) return BS_ERR_LAUNCH;
  return BS_OK;
}
template <bool RELU2>
int launch_dw_nmb(int nmb, const CUtensorMap &ta, const CUtensorMap &tc, const DwParams &P,
                  int sms, cudaStream_t st) {
  switch (nmb) {
    case 1: return launch_dw<1, RELU2>(ta, tc, P, sms, st);
    case 2: return launch_dw<2, RELU2>(ta, tc, P, sms, st);
    case 3: return launch_dw<3, RELU2>(ta, tc, P, sms, st);
    default: return launch_dw<4, RELU2>(ta, tc, P, sms, st);
  }
}
}  // namespace
}  // namespace bs

extern "C" size_t bs_gemm_unpack_dw_workspace_bytes(int64_t T, int64_t D, int64_t H) {
  if (T <= 0 || D <= 0 || H <= 0) return 0;
  const int sms = dev_sms();
  if (sms <= 0) return 0;
  const DwPlan p = dw_plan(T, D, H, sms);
  return p.ks > 1 ? (size_t)p.ks * (size_t)D * (size_t)H * sizeof(float) : 0;
}

extern "C" int bs_gemm_unpack_dw(const void *g, int64_t ldg, int64_t T, int64_t D,
                                 const void *vals, const uint8_t *bitmask,
                                 const uint32_t *prefix, const int64_t *vals_offset, int64_t H,
                                 int relu2, float k, void *C, int64_t ldc, void *workspace,
                                 size_t workspace_bytes, int32_t *status, void *stream) {
  if (T < 0 || D < 0 || H < 0) return BS_ERR_SHAPE;
  if (D == 0 || H == 0) return BS_OK;
  // (vals may be null when the tensor holds no values)
  if (!g || !C || !bitmask || !prefix || !vals_offset) return BS_ERR_ARG;
  if (ldg < D || ldc < H) return BS_ERR_SHAPE;
  if (relu2 && k != 1.0f) return BS_ERR_ARG;  // the fused square assumes k = 1
  if (T >= ((int64_t)1 << 31) || D >= ((int64_t)1 << 31) || H >= ((int64_t)1 << 31))
    return BS_ERR_TOO_LARGE;
  if ((reinterpret_cast<uintptr_t>(g) & 15) || ((ldg * 2) & 15) ||
      (reinterpret_cast<uintptr_t>(vals) & 15) || (reinterpret_cast<uintptr_t>(bitmask) & 15))
    return BS_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0) {  // empty reduction: C = 0
    for (int64_t r = 0; r < D; ++r)
      if (cudaMemsetAsync(static_cast<uint8_t *>(C) + r * ldc * 2, 0, (size_t)H * 2, st) !=
          cudaSuccess)
        return BS_ERR_LAUNCH;
    return BS_OK;
  }
  const int sms = dev_sms();
  if (sms < 2) return BS_ERR_LAUNCH;
  const DwPlan plan = dw_plan(T, D, H, sms);
  DwParams P{};
  if (plan.ks > 1) {
    const size_t need = (size_t)plan.ks * (size_t)D * (size_t)H * sizeof(float);
    if (!workspace || workspace_bytes < need) return BS_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 15) return BS_ERR_ALIGN;
    P.part = static_cast<float *>(workspace);
  }
  P.C = static_cast<uint8_t *>(C);
  P.M = D; P.N = H; P.K = T; P.ldc = ldc;
  P.ks = plan.ks;
  P.kspan = plan.kspan;
  P.mt = plan.mt;
  P.nt = plan.nt;
  P.vals = static_cast<const uint8_t *>(vals);
  P.bitmask = bitmask;
  P.prefix = prefix;
  P.vals_offset = vals_offset;
  P.grid_n = (H + kTileN - 1) / kTileN;
  P.status = status;
  P.c_tma = ((reinterpret_cast<uintptr_t>(C) & 15) == 0) && ((ldc * 2) % 16 == 0);
  CUtensorMap ta, tc;
  if (!make_map(&ta, g, T, D, ldg, 64, 64)) return BS_ERR_ALIGN;
  if (P.c_tma && !make_map(&tc, C, D, H, ldc, 64, 32)) P.c_tma = 0;
  if (!P.c_tma) tc = ta;  // unused
  int rc = relu2 ? launch_dw_nmb<true>(plan.nmb, ta, tc, P, sms, st)
                 : launch_dw_nmb<false>(plan.nmb, ta, tc, P, sms, st);
  if (rc != BS_OK || plan.ks == 1) return rc;
  const int64_t total = D * H;
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
  dw_reduce_kernel<<<(unsigned)blocks, 256, 0, st>>>(P.part, plan.ks, D, H,
                                                      static_cast<uint8_t *>(C), ldc);
  return cudaGetLastError() == cudaSuccess ? BS_OK : BS_ERR_LAUNCH;
}
