// tcgen05 (5th-generation tensor core) float32 GEMM with 3xTF32 split
// emulation, for sm_100a.
//
// Precision. fp32 has no tensor-core kind, so each operand value x is split
// into two tf32 values, hi = round_tf32(x) and lo = x - hi (exact in fp32):
//   a*b ~= hi(a)*hi(b) + hi(a)*lo(b) + lo(a)*hi(b)        (lo*lo dropped)
// Tensor-core accumulation truncates, so a long K loop into one accumulator
// drifts; instead the MMAs accumulate a *partial* over GROUP K-slices (256
// values of K) in tensor memory, and promoter warps fold each partial into
// the total with correctly rounded fp32 adds. The result has fp32-class error
// (the same order as a plain fp32 dot product).
//
// Work split. Two CTAs on a pair of SMs (a cluster of 2, cta_group::2)
// compute a 256 x 256 tile of C: each CTA stages 128 rows of A and 128 rows
// of B per K-slice and receives 128 rows x 256 columns of the accumulator in
// its own TMEM. The CTAs are persistent and walk the tiles of C in a fixed
// order. Roles per CTA (16 warps):
//   warp 0      TMA producer: fp32 slices of A and B (16 elements of K) into
//               a 6-stage shared-memory ring, K-major or M/N-major;
//   warp 1      (leader CTA) MMA issuer: 3 x 2 tcgen05.mma per slice into a
//               partial accumulator, commits that free the slot in both CTAs
//               (both warps run their loops warp-wide; one elected lane
//               issues);
//   warps 2-7   splitters, one per ring slot: warp 2+j rewrites every slice
//               landing in slot j as tf32 hi (in place) and lo (beside it),
//               then signals the leader's MMA, so six slices are split
//               concurrently and each warp's fence/arrive latency is hidden;
//   warps 8-15  promoters: read each finished partial into registers and add
//               it to the tile's running total, which lives in their
//               registers (128 values per thread); at the end of a tile the
//               epilogue (bias, activation or activation derivative, store)
//               goes from those registers through a per-warp shared-memory
//               transpose, so global loads and stores are coalesced rows.
// Tensor memory holds two partial accumulators (columns [0,256) and
// [256,512)): the MMAs of one group of K-slices run while the promoters read
// the other, so neither waits for the other, and a tile's epilogue overlaps
// the next tile's first two groups. The register split (setmaxnreg) gives
// warps 0-7 64 registers each and the promoters 192.
//
// Implicit-GEMM convolution. The same pipeline runs a convolution without
// materialising its im2col columns: the splitter warps, which rewrite every
// staged tile anyway, instead read the im2col values of the A operand
// straight from the NCHW tensor (x, or dy for the input gradient) and write
// them, split, into the swizzled shared-memory layout the MMA reads. For
// tiles up to 128 wide, four gather warps write them to tensor memory
// instead, and the MMA reads A from there (TileT, a_in_tmem). Two
// orientations: positions on M with the input channels' patches on K (the
// forward pass, and the input gradient as the forward convolution of dy with
// the flipped, transposed weight), and patches on M with positions on K (the
// weight gradient, whose B operand, dy itself, comes by a 3-D TMA copy over
// (positions, channels, images), and whose A operand has an extra row of
// ones so that the bias gradient is one more row of the product). The tile
// width BN (64, 128 or 256 columns) fits the channel count on N.
//
// Every barrier wait is bounded in time; on expiry the kernel records the
// waiting site in an error word (reported by gt_sync), stops its loops,
// waits (bounded) for its copies and MMAs in flight, frees its tensor memory
// and returns instead of hanging the GPU. No thread returns early, so the
// closing cluster barrier is always reached by every thread.
#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <type_traits>

#include "gemm.cuh"

namespace gt {

__device__ int g_tc_error = 0;

namespace tc {

constexpr int BM = 128;    // A rows per CTA (a pair covers 256)
constexpr int BK = 16;     // K elements per slice
constexpr int STAGES = 6;
constexpr int MAX_STAGES = 12;  // the deepest ring (a gathered A in tensor memory, 64-wide tiles)
// One splitter warp per ring slot: splitter w takes slices w, w + 6, ...,
// all of which land in slot w, so its waits on that slot's barrier come in
// phase order. (A barrier's parity wait cannot tell a phase from the one two
// phases later, so two warps sharing a slot could wake on stale data.)
constexpr int SPLITTERS = STAGES;
constexpr int GROUP = 16;  // K slices per promotion group
constexpr int THREADS = 512;
constexpr int SPLIT_WARP0 = 2;  // warps 2..2+SPLITTERS-1 split
constexpr int PROMOTERS = 256;
constexpr uint32_t A_BYTES = BM * BK * 4;
constexpr int PROMOTER_WARPS = PROMOTERS / 32;
constexpr int EPI_LD = 33;  // padded row of the per-warp 32 x 32 transpose (conflict-free both ways)
constexpr uint32_t EPI_BYTES = PROMOTER_WARPS * 32 * EPI_LD * 4;

// Layout of one instantiation for a tile of 256 x BN outputs (C columns BN;
// each CTA holds BN / 2 rows of B per stage and 128 lanes x BN columns of
// each of the two tensor-memory accumulators).
template <int BN, bool HALO = false>
struct Tile {
  static_assert(BN == 64 || BN == 128 || BN == 256, "tile width");
  static constexpr int BNH = BN / 2;  // B rows per CTA
  static constexpr uint32_t B_BYTES = BNH * BK * 4;
  // A hi, A lo, B hi, B lo, and (HALO) a region of A_BYTES for a gathered
  // operand's halo, so the gather writes both split planes in one pass.
  static constexpr uint32_t HALO_OFFSET = 2 * (A_BYTES + B_BYTES);
  static constexpr uint32_t STAGE_BYTES = HALO_OFFSET + (HALO ? A_BYTES : 0u);
  static constexpr uint32_t B_OFF = 2 * A_BYTES;                        // B hi (B lo follows)
  static constexpr uint32_t HALO_OFF = HALO ? HALO_OFFSET : A_BYTES;  // a gathered operand's halo
  static constexpr uint32_t A_COL0 = 0;                               // unused: A is in shared memory
  static constexpr bool NCAT = false;
  static constexpr int ACC = BN;
  static constexpr int STAGES = tc::STAGES;
  static constexpr uint32_t BAR_OFFSET = STAGES * STAGE_BYTES;
  static constexpr uint32_t EPI_OFFSET = BAR_OFFSET + 512;
  static constexpr uint32_t SMEM_BYTES = EPI_OFFSET + EPI_BYTES + 1024;  // + slack for 1024-byte alignment
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // two partial accumulators of BN columns
  static constexpr int HC = BN / 2;               // columns per promoter warp
  static constexpr int64_t TILE_ELEMS = 2 * BM * BN;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(STAGES <= MAX_STAGES && STAGES == SPLITTERS, "one splitter warp per slot");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

// Layout of an instantiation whose gathered A operand goes to tensor memory
// (tile widths 64 and 128): the two partial accumulators take columns
// 0 .. 2 ACC - 1, and ring slot s keeps its slice's A hi and A lo (16 columns
// each, lane = row, column = k, the layout the MMA reads A from tensor memory
// in) at columns A_COL0 + 32 s. Shared memory holds per slot only B's two
// planes and the halo, so the ring is as deep as the columns allow.
// NCAT (width 64): each CTA's B hi and B lo rows are adjacent, so one MMA of
// width 2 BN multiplies an A plane by both: two MMAs per K step (A hi and
// A lo against [B hi | B lo]) instead of three, whose issue bounds the
// narrow tile. An accumulator then holds each output column twice, the
// products with B hi and with B lo, which the promoters add.
template <int BN>
struct TileT {
  static_assert(BN == 64 || BN == 128, "tile width");
  static constexpr int BNH = BN / 2;
  static constexpr bool NCAT = BN == 64;
  static constexpr int ACC = NCAT ? 2 * BN : BN;  // accumulator columns per partial buffer
  static constexpr uint32_t B_BYTES = BNH * BK * 4;
  static constexpr uint32_t B_OFF = 0;
  static constexpr uint32_t HALO_OFF = 2 * B_BYTES;
  static constexpr uint32_t STAGE_BYTES = HALO_OFF + A_BYTES;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t A_COL0 = 2 * ACC;
  static constexpr int STAGES = (int)((TMEM_COLS - A_COL0) / 32) < MAX_STAGES ? (int)((TMEM_COLS - A_COL0) / 32)
                                                                              : MAX_STAGES;
  static constexpr uint32_t BAR_OFFSET = STAGES * STAGE_BYTES;
  static constexpr uint32_t EPI_OFFSET = BAR_OFFSET + 512;
  static constexpr uint32_t TAB_OFFSET = EPI_OFFSET + EPI_BYTES;  // the gather's tap table (KH * KW <= 64)
  static constexpr uint32_t SMEM_BYTES = TAB_OFFSET + 64 * 16 * 4 + 1024;
  static constexpr int HC = BN / 2;
  static constexpr int64_t TILE_ELEMS = 2 * BM * BN;
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(TAB_OFFSET % 16 == 0, "the table is read as int4");
  static_assert(A_COL0 + 32u * STAGES <= TMEM_COLS, "A slots fit the allocation");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};
constexpr int BN = 256;  // the plain GEMMs' tile width
constexpr int BNH = Tile<BN>::BNH;
constexpr uint32_t BUF_COLS = 256;
// Registers per thread after the split: warps 0-7 (TMA, MMA, splitters) and
// warps 8-15 (promoters). The launch gives every thread 65536 / 512 = 128;
// the split keeps the block's total: 256 * 64 + 256 * 192 = 256 * 128 * 2.
constexpr int REGS_LOW = 64, REGS_HIGH = 192;
static_assert(256 * REGS_LOW + 256 * REGS_HIGH <= THREADS * 128, "register split exceeds the launch's registers");
constexpr uint64_t kTimeoutNs = 2000000000ull;  // default limit, 2 s; a healthy wait takes microseconds

// Where an operand comes from. A: TMA, or gathered by the splitter warps as
// im2col values with positions on the rows (A_IM2COL_POS) or patch entries
// on the rows (A_IM2COL_CK). B: a 2-D TMA copy, a 3-D one over (positions
// per image, channels, images) whose K index is image * L + position, or two
// 2-D copies of an operand already split into tf32 planes (B_SPLIT2: hi rows
// from 0, lo rows from Gather::b_lo_row), which the splitters leave alone.
enum ASrc : int { A_TMA = 0, A_IM2COL_POS = 1, A_IM2COL_CK = 2, A_IM2COL_POS_FULL = 3 };
enum BSrc : int { B_TMA2 = 0, B_TMA3 = 1, B_SPLIT2 = 2 };

// The im2col geometry of a gathered operand (stride 1): src (N, C, H, W) read
// through KH x KW windows with the padding, L = OH * OW positions per image.
// Column k of the patch matrix is (c, kh, kw) = (k / KHW, k % KHW / KW,
// k % KW), as internal/cpu/linalg.go:122-146 lays it out. ones_row (the
// A_IM2COL_CK orientation) is a row of ones (-1: none).
//
// Per K-slice the producer copies, with one 4-D TMA load over src's
// (W, H, C, N) dimensions, the "halo" the slice needs into the stage's halo
// region (the lo plane at BN 256): box_w columns from x0 (rounded down to a
// 16-byte boundary, so the TMA's innermost coordinate stays aligned), box_h
// rows, box_c channels, box_n images, zero outside the tensor (the
// convolution's padding). The splitter warps build the slice's im2col tile
// from it in shared memory, or the gather warps in tensor memory.
//   A_IM2COL_POS: a CTA's 128 rows are 128 consecutive positions forming a
//     rectangle: rows_pi (= bh * OW) positions of each of box_n images, bh
//     output rows each. The halo holds the channels of the slice's 16 patch
//     entries.
//   A_IM2COL_CK: a slice's 16 positions form a rectangle of one image (r16
//     rows of min(OW, 16) columns); the halo holds the channels of the CTA's
//     128 patch-entry rows.
// rp is the padding rounded up to a multiple of 4: the halo's column 0 is
// input column (first output column) - rp. Every index fits 32 bits (the
// host checks).
struct Gather {
  int C = 0, H = 0, W = 0, KH = 1, KW = 1, OW = 1, pad = 0;
  int L = 1, KHW = 1, CKK = 0, ones_row = -1;
  int rp = 0, box_w = 0, box_h = 0, box_c = 0, box_n = 1;
  int bh = 1, rows_pi = 1;  // A_IM2COL_POS
  // A_IM2COL_POS with 2 x 2 pooling fused into the epilogue (EK_NCHW_POOL):
  // the CTA's rows are its positions in window order, row 4 w + k = offset k
  // (kh * 2 + kw) of 2 x 2 window w, so a window's four values sit in four
  // adjacent lanes. Set by the host for that kind; the kernel keys on EK.
  int pool2 = 0;
  // A_IM2COL_POS_FULL (set with it): the halo holds whole unpadded image
  // planes (box_w = W, box_h = H; box_c channels of box_n images from the
  // image of the tile's first position), so a tile's 128 positions need not
  // be whole rows; each row's plane offset and in-image taps are computed per
  // tile, and the padding's zeros come from those masks.
  int full = 0;
  int r16 = 1, w16 = 16;    // A_IM2COL_CK
  uint32_t halo_bytes = 0;  // box_w * box_h * box_c * box_n * 4
  int b_lo_row = 0;         // B_SPLIT2: first row of the lo plane
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t num_clusters() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// The shared::cluster address of a local shared-memory object in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Arrival on the barrier at the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ void mbar_arrive_rank(uint64_t* bar, uint32_t rank) {
  uint32_t remote = map_to_rank(smem_u32(bar), rank);
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase of `bar` with the given parity; false (and the error
// word set to `site`) once `limit_ns` has passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int site, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > limit_ns) {
      atomicCAS(&g_tc_error, 0, site);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 "version 1").
//   K-major operands: 64-byte rows (16 fp32 of K) with the 64-byte swizzle;
//     8-row groups 512 B apart (SBO); one K step (8 tf32) is +32 bytes.
//   M/N-major operands (tf32 supports only the 128-byte swizzle with 32-byte
//     atoms there): 128-byte rows of 32 M/N elements, one per k; 32-element
//     groups LBO = BK*128 bytes apart, 4-row groups 512 B apart (SBO); one K
//     step (8 rows) is +1024 bytes.
constexpr uint32_t kLayoutSw64 = 4, kLayoutSw128Atom32 = 1;
constexpr uint32_t kLboMN = BK * 128;

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for tcgen05
  d |= (uint64_t)layout << 61;
  return d;
}

template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kk) {
  return MN ? smem_desc(base + kk * 1024, kLboMN, 512, kLayoutSw128Atom32)
            : smem_desc(base + kk * 32, 16, 512, kLayoutSw64);
}

// Instruction descriptor for kind::tf32, fp32 accumulate, M = 256 (pair), N = TBN.
template <bool A_MN, bool B_MN, int TBN>
__device__ __forceinline__ uint32_t instr_desc() {
  uint32_t d = 0;
  d |= 1u << 4;                 // D format: F32
  d |= 2u << 7;                 // A format: TF32
  d |= 2u << 10;                // B format: TF32
  d |= (A_MN ? 1u : 0u) << 15;  // A major
  d |= (B_MN ? 1u : 0u) << 16;  // B major
  d |= (uint32_t)(TBN >> 3) << 17;
  d |= (uint32_t)((2 * BM) >> 4) << 24;
  return d;
}

// (The form without a disable-output-lane mask: every lane is written.)
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same MMA with A read from tensor memory at column `tmem_a` (in each CTA
// of the pair, its 128 rows on the 128 lanes; A K-major).
__device__ __forceinline__ void mma_tf32_pair_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// One lane of the converged warp (elect.sync): the producer and MMA warps run
// their loops warp-wide, so addresses and descriptors stay warp-uniform, and
// only the elected lane issues the copies, MMAs and commits.
__device__ __forceinline__ bool elect_one() {
  uint32_t e;
  asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(e));
  return e != 0;
}

// Arrives on `bar` in both CTAs of the pair once the MMAs issued so far complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

__device__ __forceinline__ void tmem_load32(uint32_t taddr, float* v) {
  uint32_t r[32];
  // Load and wait in one asm block: the registers are valid only after the wait.
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_store32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

// One warp splits n16 float4s of a staged slice in place: x -> hi = tf32(x)
// over x, lo = tf32(x - hi) into the lo plane. The tensor core reads an fp32
// operand of kind::tf32 by dropping its low 13 bits (truncation), so both
// halves are stored already rounded: lo = x - hi is exact in fp32, and
// rounding it too keeps the pair within half a tf32 ulp of lo.
__device__ __forceinline__ void split_tf32(float4* x, float4* lo, int n16, int lane) {
#pragma unroll 8
  for (int i = lane; i < n16; i += 32) {
    float4 v = x[i], h, l;
    h.x = tf32_round(v.x), h.y = tf32_round(v.y), h.z = tf32_round(v.z), h.w = tf32_round(v.w);
    l.x = tf32_round(__fsub_rn(v.x, h.x)), l.y = tf32_round(__fsub_rn(v.y, h.y));
    l.z = tf32_round(__fsub_rn(v.z, h.z)), l.w = tf32_round(__fsub_rn(v.w, h.w));
    x[i] = h;
    lo[i] = l;
  }
}

// Byte offset of element (r, k) of a K-major stage operand (128 rows of 16
// fp32, 64-byte rows, the 64-byte swizzle the TMA writes and the MMA's
// descriptor reads: the 16-byte chunk index XORed with address bits 7-8).
__device__ __forceinline__ uint32_t kmajor_offset(int r, int chunk) {
  return (uint32_t)r * 64u + ((uint32_t)(chunk ^ ((r >> 1) & 3)) << 4);
}

__device__ __forceinline__ void split_store4(uint8_t* hi, uint8_t* lo, uint32_t off, float a, float b, float c,
                                             float d) {
  float4 h, l;
  h.x = tf32_round(a), h.y = tf32_round(b), h.z = tf32_round(c), h.w = tf32_round(d);
  l.x = tf32_round(__fsub_rn(a, h.x)), l.y = tf32_round(__fsub_rn(b, h.y));
  l.z = tf32_round(__fsub_rn(c, h.z)), l.w = tf32_round(__fsub_rn(d, h.w));
  *(float4*)(hi + off) = h;
  *(float4*)(lo + off) = l;
}

// A_IM2COL_POS: rows 0..rows-1 of this CTA's A block are output positions
// (the block starts at a rectangle of the output), columns k0 .. k0+15 patch
// entries (c, kh, kw). Lane l fills rows l, l+32, l+64, l+96, whose halo
// offsets hb[] pos_rows() computes once per kernel (the block's layout in the
// halo is the same for every tile). Each chunk of four entries of a row goes
// to the hi plane as one 16-byte store of raw values (conflict-free under the
// swizzle); the warp's halo reads are 32 consecutive positions. Entries past
// C*KH*KW are zero; taps in the padding read the halo's zero fill
// (internal/cpu/linalg.go:130-139).
template <bool POOL2>
__device__ __forceinline__ int pos_row(const Gather& g, int r) {
  const int plane = g.box_w * g.box_h;
  int n, oh, ow;
  if constexpr (POOL2) {
    const int w = r >> 2, k = r & 3, per = g.rows_pi >> 2, pw = g.OW >> 1;
    n = w / per;
    const int rem = w - n * per, pr = rem / pw, pc = rem - pr * pw;
    oh = 2 * pr + (k >> 1), ow = 2 * pc + (k & 1);
  } else {
    n = r / g.rows_pi;
    const int rem = r - n * g.rows_pi;
    oh = rem / g.OW, ow = rem - oh * g.OW;
  }
  return n * g.box_c * plane + oh * g.box_w + ow + g.rp - g.pad;
}

template <bool POOL2>
__device__ __forceinline__ void pos_rows(const Gather& g, int lane, int (&hb)[4]) {
#pragma unroll
  for (int i = 0; i < 4; i++) hb[i] = pos_row<POOL2>(g, lane + 32 * i);
}

// pos_rows for A_IM2COL_POS_FULL: row r of the tile starting at position
// a_row (window-major when POOL2: index 4 w + k = offset k of window w, windows
// in pooled order, images contiguous). The halo holds box_n unpadded image
// planes (H x W) of box_c channels from the image of the tile's first
// position: hb is the offset of the row's patch origin (oh - pad, ow - pad),
// mk the taps (kh, kw) that fall inside the image. A row past M gets no
// taps: it only reaches rows of C that are never stored.
template <bool POOL2>
__device__ __forceinline__ void pos_row_full(const Gather& g, int a_row, int64_t M, int r, int& hb, int& mk) {
  const int plane = g.box_w * g.box_h, n0 = a_row / g.L;
  const int p = a_row + r;
  hb = 0, mk = 0;
  if (p >= M) return;
  const int n = p / g.L, rem = p - n * g.L;
  int oh, ow;
  if constexpr (POOL2) {
    const int w = rem >> 2, k = rem & 3, pw = g.OW >> 1, ph = w / pw, pc = w - ph * pw;
    oh = 2 * ph + (k >> 1), ow = 2 * pc + (k & 1);
  } else {
    oh = rem / g.OW, ow = rem - oh * g.OW;
  }
  const int ih = oh - g.pad, iw = ow - g.pad;
  hb = (n - n0) * g.box_c * plane + ih * g.box_w + iw;
  uint32_t m = 0;
  for (int kh = 0; kh < g.KH; kh++) {
    if ((unsigned)(ih + kh) >= (unsigned)g.box_h) continue;
    for (int kw = 0; kw < g.KW; kw++)
      if ((unsigned)(iw + kw) < (unsigned)g.box_w) m |= 1u << (kh * g.KW + kw);
  }
  mk = (int)m;
}

template <bool POOL2>
__device__ __forceinline__ void pos_rows_full(const Gather& g, int a_row, int64_t M, int lane, int (&hb)[4],
                                              int (&mk)[4]) {
#pragma unroll
  for (int i = 0; i < 4; i++) pos_row_full<POOL2>(g, a_row, M, lane + 32 * i, hb[i], mk[i]);
}

// The tap table of a gathered operand in tensor memory. A slice's 16 patch
// entries start at entry k0; with m = k0 % KHW, entry j is (channel
// k0 / KHW + dc, tap) for t = m + j, dc = t / KHW, tap = t % KHW, and
// tab[16 m + j] packs tap << 16 | (dc * plane + kh * box_w + kw), its offset
// in the slice's halo (below 2^16: a halo holds at most 2048 values). Built
// once per kernel, so the gather itself needs no index arithmetic.
__device__ __forceinline__ void build_tap_table(const Gather& g, int* tab, int tid, int nthreads) {
  const int plane = g.box_w * g.box_h;
  for (int i = tid; i < g.KHW * 16; i += nthreads) {
    const int m = i >> 4, t = m + (i & 15), dc = t / g.KHW, tap = t - dc * g.KHW;
    const int kh = tap / g.KW, kw = tap - kh * g.KW;
    tab[i] = (tap << 16) | (dc * plane + kh * g.box_w + kw);
  }
}

__device__ __forceinline__ float ld_shared_f32(uint32_t addr) {
  float x;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"(addr) : "memory");
  return x;
}

__device__ __forceinline__ int4 ld_shared_v4(uint32_t addr) {
  int4 v;
  asm volatile("ld.shared.v4.s32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

// A gathered operand in tensor memory: the lane's own row (hb, mk as above;
// live false for a row past M, which gets zeros) over the slice's 16 patch
// entries from k0, whose table entries start at shared address `tab16`,
// split into v[0..15] = hi and v[16..31] = lo, the order of the slot's 32
// columns. The warp's halo reads are 32 consecutive positions.
template <bool FULL>
__device__ __forceinline__ void gather_row_split(const Gather& g, uint32_t halo, uint32_t tab16, bool live, int k0,
                                                 int hb, int mk, float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int4 q = ld_shared_v4(tab16 + 16 * i);
    const int e[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int kk = 4 * i + j;
      bool take = live && k0 + kk < g.CKK;
      if constexpr (FULL) take = take && ((mk >> (e[j] >> 16)) & 1);
      const float x = take ? ld_shared_f32(halo + 4u * (uint32_t)(hb + (e[j] & 0xFFFF))) : 0.0f;
      const float h = tf32_round(x);
      v[kk] = h;
      v[16 + kk] = tf32_round(__fsub_rn(x, h));
    }
  }
}

__device__ __forceinline__ void store_row4(uint8_t* hi, uint8_t* lo, uint32_t off, float a, float b, float c,
                                           float d) {
  if (lo)
    split_store4(hi, lo, off, a, b, c, d);
  else
    *(float4*)(hi + off) = make_float4(a, b, c, d);
}

// lo NULL: raw values into the hi plane (split in place afterwards); else the
// split planes directly.
// FULL (A_IM2COL_POS_FULL): the halo holds unpadded image planes, hb[i] is
// the plane offset of row i's patch origin (negative inside the padding) and
// bit kh * KW + kw of mk[i] says whether that tap lies inside the image (the
// others are the padding's zeros and are not read).
template <bool FULL>
__device__ __forceinline__ void gather_pos(const Gather& g, uint8_t* hi, uint8_t* lo, const float* halo, int rows,
                                           int k0, int lane, const int (&hb)[4], const int (&mk)[4]) {
  // Lane j < 16 packs entry k0 + j as the tap table does (tap << 16 | halo
  // offset); the warp reads entry kk from lane kk, so the loads need no
  // serial index arithmetic.
  int my_e;
  {
    const int plane = g.box_w * g.box_h, m = k0 % g.KHW, t = m + (lane & 15), dc = t / g.KHW;
    const int tap = t - dc * g.KHW, kh = tap / g.KW, kw = tap - kh * g.KW;
    my_e = (tap << 16) | (dc * plane + kh * g.box_w + kw);
  }
  const uint32_t hs = smem_u32(halo);
#pragma unroll 1
  for (int c4 = 0; c4 < 4; c4++) {
    float v[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      const int e = __shfl_sync(0xffffffffu, my_e, 4 * c4 + kk);
      const bool kin = k0 + 4 * c4 + kk < g.CKK;
      const int koff = e & 0xFFFF;
      if constexpr (FULL) {
        const int tap = e >> 16;
#pragma unroll
        for (int i = 0; i < 4; i++)
          v[i][kk] = kin && ((mk[i] >> tap) & 1) ? ld_shared_f32(hs + 4u * (uint32_t)(hb[i] + koff)) : 0.0f;
      } else {
#pragma unroll
        for (int i = 0; i < 4; i++) v[i][kk] = kin ? ld_shared_f32(hs + 4u * (uint32_t)(hb[i] + koff)) : 0.0f;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int r = lane + 32 * i;
      if (r < rows) store_row4(hi, lo, kmajor_offset(r, c4), v[i][0], v[i][1], v[i][2], v[i][3]);
    }
  }
}

// A_IM2COL_CK: rows 0..rows-1 of this CTA's A block are patch entries
// row0 + r = (c, kh, kw), columns the slice's 16 positions. Lane l fills rows
// l, l+32, l+64, l+96: ck_rows() gives, once per tile, each row's offset in
// the halo (channel relative to the block's first) and its kind (gathered,
// zero past C*KH*KW, or the row of ones that makes that row of the product
// the bias gradient). A row's 16 positions go out as four 16-byte stores.
__device__ __forceinline__ void ck_row(const Gather& g, int row0, int r, int& koff, int& kind) {
  const int plane = g.box_w * g.box_h, c_lo = row0 / g.KHW;
  const int ck = row0 + r;
  const int c = ck / g.KHW, rem = ck - c * g.KHW, kh = rem / g.KW, kw = rem - kh * g.KW;
  koff = (c - c_lo) * plane + kh * g.box_w + kw + g.rp - g.pad;
  kind = ck < g.CKK ? 1 : ck == g.ones_row ? 2 : 0;
}

__device__ __forceinline__ void ck_rows(const Gather& g, int row0, int lane, int (&koff)[4], int (&kind)[4]) {
#pragma unroll
  for (int i = 0; i < 4; i++) ck_row(g, row0, lane + 32 * i, koff[i], kind[i]);
}

// A_IM2COL_CK in tensor memory: the lane's own patch row (koff, kind from
// ck_row) over the slice's 16 positions, split into v[0..15] = hi and
// v[16..31] = lo. The slice's positions are rows of w16 (a power of two)
// positions box_w apart in the halo, so each offset is independent of the
// others. Only gathered rows (kind 1) read the halo.
__device__ __forceinline__ void gather_ck_row_split(const Gather& g, uint32_t halo, int koff, int kind,
                                                    float (&v)[32]) {
  const int lw = __ffs(g.w16) - 1;
  const float fill = kind == 2 ? 1.0f : 0.0f;
#pragma unroll
  for (int p = 0; p < 16; p++) {
    const int off = (p >> lw) * g.box_w + (p & (g.w16 - 1));
    const float x = kind == 1 ? ld_shared_f32(halo + 4u * (uint32_t)(koff + off)) : fill;
    const float h = tf32_round(x);
    v[p] = h;
    v[16 + p] = tf32_round(__fsub_rn(x, h));
  }
}

__device__ __forceinline__ void gather_ck(const Gather& g, uint8_t* hi, uint8_t* lo, const float* halo, int rows,
                                          int lane, const int (&koff)[4], const int (&kind)[4]) {
#pragma unroll 1
  for (int i = 0; i < 4; i++) {
    const int r = lane + 32 * i;
    if (r >= rows) break;
    float v[16];
    if (kind[i] == 1) {
      int oh = 0, ow = 0;
#pragma unroll
      for (int p = 0; p < 16; p++) {
        v[p] = halo[koff[i] + oh * g.box_w + ow];
        if (++ow == g.w16) ow = 0, ++oh;
      }
    } else {
      const float f = kind[i] == 2 ? 1.0f : 0.0f;
#pragma unroll
      for (int p = 0; p < 16; p++) v[p] = f;
    }
#pragma unroll
    for (int c4 = 0; c4 < 4; c4++)
      store_row4(hi, lo, kmajor_offset(r, c4), v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
  }
}

// Epilogue kinds: each kernel instantiation carries only the code of its
// kind. The promoters' code shares the SM's instruction cache with the MMA
// issuer and the splitters, and large unrolled epilogues measurably slowed
// the whole pipeline, so every kind keeps its unrolled part small.
enum EpiKind : int {
  EK_PLAIN = 0,      // C stored row-major
  EK_BIAS_RELU = 1,  // + bias[n] (optional), then ReLU (optional): Linear forward
  EK_MASK = 2,       // * act'(mask[m][n]): the dX of a Linear after an activation
  EK_CONV = 3,       // + bias[m] (optional), then ReLU (optional), stored in NCHW order: Conv2d forward
  EK_GENERIC = 4,    // anything else (tanh / sigmoid forward)
  EK_MASKBITS = 5,   // * Step from a ReLU bit mask: the dX of a Linear after a ReLU
  EK_NCHW_POS = 6,   // + bias[n] (optional), ReLU (optional), m = position, n = channel, stored NCHW:
                     // an implicit-GEMM convolution's forward pass or input gradient
  EK_COLMAJOR = 7,   // stored transposed, with the bias-gradient row: a convolution's weight gradient
  EK_NCHW_POOL = 8,  // EK_NCHW_POS followed by 2 x 2 / stride-2 max pooling: only the pooled values
                     // and their first-max offsets are stored (rows in window order, Gather::pool2)
};

inline int epi_kind(const Epi<float>& e, int64_t n_cols) {
  if (e.col_major) return !e.bias && e.act == GT_ACT_NONE && !e.dmask && !e.dbits && !e.bits_out ? EK_COLMAJOR : -2;
  if (e.pos_major && e.pool_idx)
    return e.nchw_L > 0 && !e.bias_by_row && (e.act == GT_ACT_NONE || e.act == GT_ACT_RELU) && !e.dmask &&
                   !e.dbits && !e.bits_out
               ? EK_NCHW_POOL
               : -2;
  if (e.pos_major)
    return e.nchw_L > 0 && !e.bias_by_row && (e.act == GT_ACT_NONE || e.act == GT_ACT_RELU) && !e.dmask &&
                   !e.dbits && !e.bits_out
               ? EK_NCHW_POS
               : -2;
  const bool rowmajor = e.nchw_L == 0;
  if (e.bits_out)  // only this kind writes the bit mask
    return !e.bias_by_row && (e.act == GT_ACT_NONE || e.act == GT_ACT_RELU) && !e.dmask && !e.dbits && rowmajor
               ? EK_BIAS_RELU
               : -1;
  if (e.dbits) return !e.bias && e.act == GT_ACT_NONE && !e.dmask && rowmajor ? EK_MASKBITS : EK_GENERIC;
  if (!e.bias && e.act == GT_ACT_NONE && !e.dmask && rowmajor) return EK_PLAIN;
  if (!e.bias_by_row && (e.act == GT_ACT_NONE || e.act == GT_ACT_RELU) && !e.dmask && rowmajor) return EK_BIAS_RELU;
  if (!e.bias && e.act == GT_ACT_NONE && e.dmask && rowmajor) return EK_MASK;
  if ((!e.bias || e.bias_by_row) && (e.act == GT_ACT_NONE || e.act == GT_ACT_RELU) && !e.dmask && !rowmajor &&
      e.nchw_L < (1ll << 31) && n_cols < (1ll << 31))
    return EK_CONV;  // positions fit 32-bit arithmetic
  return EK_GENERIC;
}

// Finishes one 32 x 32 block of C held in the warp's transpose buffer: lane l
// owns column n of rows m0 .. m0+31, so each row's access is 128 contiguous
// bytes. Same operations, in the same order, as Epi::store.
template <int EK>
__device__ __forceinline__ void epilogue_block(const Epi<float>& epi, const GemmShape& s, float* xpose, int lane,
                                               int64_t m0, int64_t n) {
  const int rows = (int)(s.M - m0 < 32 ? s.M - m0 : 32);
  float* op = epi.out + m0 * epi.ldc + n;
  if (n >= s.N) return;
  float cs = 0.0f;  // column partial sum of the stored values (Epi::colsum_ws)
  if (EK == EK_PLAIN) {
#pragma unroll 4
    for (int r = 0; r < rows; r++) {
      const float v = xpose[r * EPI_LD + lane];
      op[r * epi.ldc] = v;
      cs = __fadd_rn(cs, v);
    }
  } else if (EK == EK_BIAS_RELU) {
    // With a bit mask, this lane's column of the block (m0 is a multiple of
    // 32) becomes one word: bit r = (row r's value > 0).
    const float b = epi.bias ? __ldg(epi.bias + n) : 0.0f;
    const bool relu = epi.act == GT_ACT_RELU;
    uint32_t w = 0;
#pragma unroll 4
    for (int r = 0; r < rows; r++) {
      float v = xpose[r * EPI_LD + lane];
      if (epi.bias) v = __fadd_rn(v, b);
      if (relu) v = go_max(v, 0.0f);
      op[r * epi.ldc] = v;
      w |= (uint32_t)(v > 0.0f) << r;
    }
    if (epi.bits_out && rows > 0) epi.bits_out[(m0 >> 5) * epi.ldw + n] = w;
  } else if (EK == EK_MASKBITS) {
    // One word holds this column's factor for all 32 rows of the block: 4
    // bytes per lane instead of 128 bytes of activations.
    const uint32_t w = rows > 0 ? __ldg(epi.dbits + (m0 >> 5) * epi.ldw + n) : 0u;
#pragma unroll 4
    for (int r = 0; r < rows; r++) {
      const float v = __fmul_rn(xpose[r * EPI_LD + lane], ((w >> r) & 1u) ? 1.0f : 0.0f);
      op[r * epi.ldc] = v;
      cs = __fadd_rn(cs, v);
    }
  } else if (EK == EK_MASK) {
    // The mask values of 8 rows are requested before any is used.
    const float* mp = epi.dmask + m0 * epi.ldm + n;
#pragma unroll 1
    for (int r0 = 0; r0 < 32; r0 += 8) {
      float mask[8];
#pragma unroll
      for (int r = 0; r < 8; r++) mask[r] = r0 + r < rows ? __ldg(mp + (r0 + r) * epi.ldm) : 0.0f;
#pragma unroll
      for (int r = 0; r < 8; r++)
        if (r0 + r < rows) {
          const float v = act_bwd(epi.dact, xpose[(r0 + r) * EPI_LD + lane], mask[r]);
          op[(r0 + r) * epi.ldc] = v;
          cs = __fadd_rn(cs, v);
        }
    }
  } else if (EK == EK_CONV) {
    // C(m, n) -> out[((n / L) * M + m) * L + n % L]: a warp's row is 32
    // consecutive positions of one channel plane (image boundaries aside).
    const uint32_t L32 = (uint32_t)epi.nchw_L, img = (uint32_t)n / L32;
    const int64_t L = epi.nchw_L;
    float* base = epi.out + (int64_t)img * epi.nchw_M * L + ((uint32_t)n - img * L32);
    const bool relu = epi.act == GT_ACT_RELU;
#pragma unroll 4
    for (int r = 0; r < rows; r++) {
      const int64_t m = m0 + r;
      float v = xpose[r * EPI_LD + lane];
      if (epi.bias) v = __fadd_rn(v, __ldg(epi.bias + m));
      if (relu) v = go_max(v, 0.0f);
      base[m * L] = v;
    }
  } else {
#pragma unroll 1
    for (int r = 0; r < rows; r++) epi.store(m0 + r, n, xpose[r * EPI_LD + lane]);
  }
  if (EK == EK_PLAIN || EK == EK_MASK || EK == EK_MASKBITS)
    if (epi.colsum_ws && rows > 0) epi.colsum_ws[(m0 >> 5) * epi.ldcs + n] = cs;
}

// How a launch covers its tiles: tiles [0, whole) as single units over all
// of K, the remaining tiles in `splits` units each over consecutive K ranges.
// A split unit stores its partial 256 x 256 tile in the workspace; a second
// kernel adds a tile's partials in split order and applies the epilogue.
struct SplitPlan {
  int whole = 0;
  int splits = 1;
  float* ws = nullptr;  // [splits][tiles - whole][256 * 256]
  uint64_t wait_limit_ns = kTimeoutNs;  // every barrier wait gives up after this long
  // Test hook (gt_debug_tc_withhold_arrive): the leader CTA's splitter of ring
  // slot 0 withholds its arrival for the first slice, so the MMA issuer's wait
  // for that slice runs out and the kernel takes its error path.
  int withhold_arrive = 0;
};

constexpr int64_t TILE_ELEMS = 2 * BM * BN;

// Work unit u: tile t over K-slices [kb, ke). Returns the split index, or -1
// for a whole tile. The splits of one tile are (tiles - whole) units apart,
// so the units running at the same time share operand panels of one K range.
__device__ __forceinline__ int unit_of(int u, int tiles, const SplitPlan& sp, int num_k, int& t, int& kb, int& ke) {
  if (u < sp.whole) {
    t = u, kb = 0, ke = num_k;
    return -1;
  }
  const int rest = tiles - sp.whole, v = u - sp.whole;
  const int sidx = v / rest;
  t = sp.whole + (v - sidx * rest);
  kb = (int)((int64_t)sidx * num_k / sp.splits);
  ke = (int)((int64_t)(sidx + 1) * num_k / sp.splits);
  return sidx;
}

struct Shared {
  uint64_t full[MAX_STAGES];   // TMA -> splitters (local)
  uint64_t split[MAX_STAGES];  // splitters of both CTAs -> leader's MMA
  uint64_t empty[MAX_STAGES];  // MMA -> producers of both CTAs
  uint64_t pfull[2];       // MMA -> promoters of both CTAs: partial buffer b is complete
  uint64_t pempty[2];      // promoter warps of both CTAs -> leader's MMA: buffer b was read
  uint64_t mma_done;       // leader: every MMA issued has completed
  uint32_t tmem_base;
  int failed;
};

// Moves the promoters' 32-column chunk J of the running total into the warp's
// transpose buffer (lane = row): the switch below keeps register indices
// static in a loop that is not unrolled, so the block's code exists once.
template <int J, int N>
__device__ __forceinline__ void xpose_chunk(float* xpose, const float (&tot)[N], int lane) {
  if constexpr (32 * J < N) {
#pragma unroll
    for (int i = 0; i < 32; i++) xpose[lane * EPI_LD + i] = tot[32 * J + i];
  }
}

// A gathered operand has its own halo region when the stage still fits six
// times in shared memory (tile widths up to 128); at 256 the halo lands in the
// A lo plane and the gather's raw values are split in place afterwards.
template <int TBN, int AS>
constexpr bool halo_region() {
  return AS != A_TMA && TBN <= 128;
}

// A position-gathered operand (A_IM2COL_POS, A_IM2COL_POS_FULL) of a tile up
// to 128 wide goes to tensor memory: four gather warps (one per lane quarter)
// write each slice's split rows with tcgen05.st, the MMA reads A from there
// and B from shared memory. Shared memory then carries no A planes, whose
// stores and the MMAs' reads of them (three reads of A per K step) bound
// these tiles on the shared-memory path.
template <int TBN, int AS>
constexpr bool a_in_tmem() {
  return AS != A_TMA && TBN <= 128;
}

template <int TBN, int AS>
using LayoutOf = std::conditional_t<a_in_tmem<TBN, AS>(), TileT<(TBN > 128 ? 128 : TBN)>,
                                    Tile<TBN, halo_region<TBN, AS>()>>;
constexpr int GATHER_WARP0 = 4;  // warps 4..7 (lane quarters 0..3) gather into tensor memory

template <bool A_MN, bool B_MN, int EK, int TBN, int AS, int BS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_tf32x3_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            GemmShape s, Epi<float> epi, SplitPlan sp, Gather ga) {
  constexpr bool HSEP = halo_region<TBN, AS>();
  constexpr bool ATM = a_in_tmem<TBN, AS>();
  using TL = LayoutOf<TBN, AS>;
  constexpr bool NCAT = TL::NCAT;
  constexpr int ACC = TL::ACC;
  // Slices per barrier round: with A in tensor memory two ring slots fill,
  // gather and free together (one wait and one commit per two slices: the
  // single MMA thread's fixed costs per round bound the narrow tiles).
  constexpr int SS = ATM ? 2 : 1;
  constexpr int NBAR = TL::STAGES / SS;
  static_assert(TL::STAGES % SS == 0 && GROUP % SS == 0, "whole rounds; groups start a round");
  constexpr int HC = TL::HC;
  constexpr int STAGES = TL::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  Shared* sh = (Shared*)(smem + TL::BAR_OFFSET);
  volatile int* failed = &sh->failed;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int num_k = (int)((s.K + BK - 1) / BK);
  const int m_tiles = (int)((s.M + 2 * BM - 1) / (2 * BM));
  const int n_tiles = (int)((s.N + TBN - 1) / TBN);
  const int tiles = m_tiles * n_tiles;
  const int units = sp.whole + (tiles - sp.whole) * sp.splits;
  const int pair = (int)cluster_id(), pairs = (int)num_clusters();

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; i++) {
      mbar_init(&sh->full[i], 1);
      mbar_init(&sh->split[i], ATM ? 2 * 4 : 2 * 32);  // per CTA: a splitter warp's lanes, or lane 0 of 4 gather warps
      mbar_init(&sh->empty[i], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&sh->pfull[b], 1);
      mbar_init(&sh->pempty[b], 2 * PROMOTER_WARPS);  // one arrival per promoter warp per CTA
    }
    mbar_init(&sh->mma_done, 1);
    sh->failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // both CTAs of the pair allocate together
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh->tmem_base)),
                 "r"(TL::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before anyone signals them
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  // Whole warpgroups change their register allocation together, each in
  // its own branch: code that both paths reach is held to the lower limit.
  if (warp < 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_LOW));
    if (warp == 0) {
      {  // ---- TMA producer (both CTAs): the warp runs the loop, the elected lane issues
        const bool issuer = elect_one();
        int it = 0, issued_to = 0;  // barrier rounds (SS slices each)
        for (int u = pair; u < units && !__shfl_sync(0xffffffffu, *failed, 0); u += pairs) {
          int t, kb, ke;
          unit_of(u, tiles, sp, num_k, t, kb, ke);
          const int mt = t / n_tiles, nt = t % n_tiles;
          const int a_row = mt * 2 * BM + (int)rank * BM;
          const int b_row = nt * TBN + (int)rank * TL::BNH;
          for (int kt = kb; kt < ke; kt += SS, it++) {
            const int nb = it % NBAR, n_in = ke - kt < SS ? ke - kt : SS;
            if (!__all_sync(0xffffffffu, mbar_wait(&sh->empty[nb], ((it / NBAR) & 1) ^ 1, 1, sp.wait_limit_ns))) {
              if (lane == 0) *failed = 1;
              break;
            }
            if (issuer) {
              uint64_t* bar = &sh->full[nb];
              mbar_expect_tx(bar, (uint32_t)n_in * ((AS == A_TMA ? A_BYTES : ga.halo_bytes) +
                                                    (BS == B_SPLIT2 ? 2u : 1u) * TL::B_BYTES));
              for (int i = 0; i < n_in; i++) {
                const int st = nb * SS + i;
                uint8_t* a_hi = smem + st * TL::STAGE_BYTES;
                uint8_t* b_hi = a_hi + TL::B_OFF;
                const int k0 = (kt + i) * BK;
                if constexpr (AS == A_IM2COL_POS) {  // the halo of this block's positions, the slice's channels
                  const int n0 = a_row / ga.L, oh0 = (a_row - n0 * ga.L) / ga.OW;
                  tma_load_4d(a_hi + TL::HALO_OFF, &tmA, bar, -ga.rp, oh0 - ga.pad, k0 / ga.KHW, n0);
                } else if constexpr (AS == A_IM2COL_POS_FULL) {  // whole planes: the slice's channels, box_n images
                  tma_load_3d(a_hi + TL::HALO_OFF, &tmA, bar, 0, k0 / ga.KHW, a_row / ga.L);
                } else if constexpr (AS == A_IM2COL_CK) {  // the halo of the slice's positions, this block's channels
                  const int n = k0 / ga.L, l0 = k0 - n * ga.L, oh0 = l0 / ga.OW, ow0 = l0 - oh0 * ga.OW;
                  tma_load_4d(a_hi + TL::HALO_OFF, &tmA, bar, ow0 - ga.rp, oh0 - ga.pad, a_row / ga.KHW, n);
                }
                if constexpr (AS == A_TMA) {
                  if (A_MN) {
#pragma unroll
                    for (int j = 0; j < BM / 32; j++) tma_load_2d(a_hi + j * kLboMN, &tmA, bar, a_row + 32 * j, k0);
                  } else {
                    tma_load_2d(a_hi, &tmA, bar, k0, a_row);
                  }
                }
                if constexpr (BS == B_TMA3) {  // K index = image * L + position
                  const int img = k0 / ga.L;
                  tma_load_3d(b_hi, &tmB, bar, k0 - img * ga.L, b_row, img);
                } else if constexpr (BS == B_SPLIT2) {  // both planes, already split
                  tma_load_2d(b_hi, &tmB, bar, k0, b_row);
                  tma_load_2d(b_hi + TL::B_BYTES, &tmB, bar, k0, ga.b_lo_row + b_row);
                } else if (B_MN) {
#pragma unroll
                  for (int j = 0; j < TL::BNH / 32; j++) tma_load_2d(b_hi + j * kLboMN, &tmB, bar, b_row + 32 * j, k0);
                } else {
                  tma_load_2d(b_hi, &tmB, bar, k0, b_row);
                }
              }
            }
            __syncwarp();
            issued_to = it + 1;
          }
        }
        if (__shfl_sync(0xffffffffu, *failed, 0)) {  // let copies in flight land before the CTA tears down
          for (int i = issued_to > NBAR ? issued_to - NBAR : 0; i < issued_to; i++)
            mbar_wait(&sh->full[i % NBAR], (i / NBAR) & 1, 5, kTimeoutNs);  // copies land in microseconds
        }
      }
    } else if (warp == 1) {
      if (leader) {  // ---- MMA issuer (leader CTA only): the warp runs the loop, the elected lane issues
        const bool issuer = elect_one();
        const uint32_t idesc = instr_desc<A_MN, B_MN, NCAT ? 2 * TBN : TBN>();
        // Descriptors of slot 0's planes; another slot or K step only moves
        // the start address (bits 0-13, in 16-byte units; shared addresses
        // stay below 256 KB, so the sum never carries out of the field).
        const uint64_t adesc0 = operand_desc<A_MN>(smem_u32(smem), 0);
        const uint64_t bdesc0 = operand_desc<B_MN>(smem_u32(smem) + TL::B_OFF, 0);
        int it = 0, group = 0;
        bool stop = false;
        for (int u = pair; u < units && !stop; u += pairs) {
          int t, kb, ke;
          unit_of(u, tiles, sp, num_k, t, kb, ke);
          for (int kt = kb; kt < ke; kt += SS, it++) {
            const int nb = it % NBAR, n_in = ke - kt < SS ? ke - kt : SS;
            if (!__all_sync(0xffffffffu, mbar_wait(&sh->split[nb], (it / NBAR) & 1, 3, sp.wait_limit_ns))) {
              stop = true;
              break;
            }
            tc_fence_after();
            for (int i = 0; i < n_in; i++) {
              const int kq = kt + i, st = nb * SS + i;
              const bool group_start = (kq - kb) % GROUP == 0;  // GROUP is a multiple of SS
              const uint32_t buf = (uint32_t)(group & 1);
              if (group_start) {  // the promoters must have read this buffer's previous partial
                if (!__all_sync(0xffffffffu,
                                mbar_wait(&sh->pempty[buf], ((group >> 1) & 1) ^ 1, 2, sp.wait_limit_ns))) {
                  stop = true;
                  break;
                }
                tc_fence_after();
              }
              const uint64_t slot = (uint64_t)((st * TL::STAGE_BYTES) >> 4);
              const uint32_t d = tmem + buf * ACC;
              // the slice's operands, computed by the whole warp (uniform)
              uint64_t dbh[BK / 8], dbl[BK / 8], dah[BK / 8], dal[BK / 8];
              uint32_t tah[BK / 8], tal[BK / 8];
#pragma unroll
              for (int kk = 0; kk < BK / 8; kk++) {
                dbh[kk] = bdesc0 + slot + (uint64_t)((B_MN ? kk * 1024 : kk * 32) >> 4);
                dbl[kk] = dbh[kk] + (TL::B_BYTES >> 4);
                dah[kk] = adesc0 + slot + (uint64_t)((A_MN ? kk * 1024 : kk * 32) >> 4);
                dal[kk] = dah[kk] + (A_BYTES >> 4);
                // A in tensor memory: hi at the slot's columns 0-15, lo at
                // 16-31, 8 columns per K step
                tah[kk] = tmem + TL::A_COL0 + 32 * st + 8 * kk;
                tal[kk] = tah[kk] + 16;
              }
              if (issuer) {
#pragma unroll
                for (int kk = 0; kk < BK / 8; kk++) {
                  const uint32_t acc0 = (group_start && kk == 0) ? 0u : 1u;
                  if constexpr (NCAT) {  // each A plane against [B hi | B lo] from dbh: the CTA's 2 BNH rows
                    mma_tf32_pair_tmem_a(d, tal[kk], dbh[kk], idesc, acc0);
                    mma_tf32_pair_tmem_a(d, tah[kk], dbh[kk], idesc, 1u);
                  } else if constexpr (ATM) {
                    mma_tf32_pair_tmem_a(d, tal[kk], dbh[kk], idesc, acc0);
                    mma_tf32_pair_tmem_a(d, tah[kk], dbl[kk], idesc, 1u);
                    mma_tf32_pair_tmem_a(d, tah[kk], dbh[kk], idesc, 1u);
                  } else {
                    mma_tf32_pair(d, dal[kk], dbh[kk], idesc, acc0);
                    mma_tf32_pair(d, dah[kk], dbl[kk], idesc, 1u);
                    mma_tf32_pair(d, dah[kk], dbh[kk], idesc, 1u);
                  }
                }
              }
              __syncwarp();
              if ((kq - kb) % GROUP == GROUP - 1 || kq == ke - 1) {
                if (issuer) mma_commit_pair(&sh->pfull[buf]);
                __syncwarp();
                group++;
              }
            }
            if (stop) break;
            if (issuer) mma_commit_pair(&sh->empty[nb]);  // frees the round's slots in both CTAs
            __syncwarp();
          }
        }
        if (stop && lane == 0) *failed = 1;
        // Every MMA must be complete before the pair frees its tensor memory
        // (the commit tracks the issuing lane's MMAs).
        if (issuer)
          asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(&sh->mma_done))
                       : "memory");
        __syncwarp();
        mbar_wait(&sh->mma_done, 0, 6, kTimeoutNs);
      }
    } else if (warp >= SPLIT_WARP0 && warp < SPLIT_WARP0 + SPLITTERS) {
      if constexpr (ATM) {
        // ---- gather warps (both CTAs): warp GATHER_WARP0 + q builds rows
        // 32 q .. 32 q + 31 of every slice's A block in its lane quarter of
        // tensor memory (lane = row), at the slot's 32 columns; warps 2-3
        // have no part.
        if (warp >= GATHER_WARP0) {
          const int q = warp & 3, r = 32 * q + lane;
          const uint32_t a_lanes = tmem + ((uint32_t)(32 * q) << 16) + TL::A_COL0;
          int* tab = (int*)(smem + TL::TAB_OFFSET);
          if constexpr (AS != A_IM2COL_CK) {  // (a weight gradient's rows carry their own offsets)
            build_tap_table(ga, tab, r, 128);
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the four gather warps
          }
          const uint32_t tab_base = smem_u32(tab);
          const int r16 = 16 % ga.KHW;
          int it = 0, hb = 0, mk = 0;
          bool stop = false;
          if constexpr (AS == A_IM2COL_POS) hb = pos_row<EK == EK_NCHW_POOL>(ga, r);
          for (int u = pair; u < units && !stop; u += pairs) {
            int t, kb, ke;
            unit_of(u, tiles, sp, num_k, t, kb, ke);
            const int a_row = (t / n_tiles) * 2 * BM + (int)rank * BM;
            if constexpr (AS == A_IM2COL_POS_FULL) pos_row_full<EK == EK_NCHW_POOL>(ga, a_row, s.M, r, hb, mk);
            if constexpr (AS == A_IM2COL_CK) ck_row(ga, a_row, r, hb, mk);  // offset and kind of the patch row
            const bool live = (int64_t)a_row + r < s.M;  // a row past M gets zeros
            int m = (kb * BK) % ga.KHW;                   // the slice's first entry's tap
            for (int kt = kb; kt < ke; kt += SS, it++) {
              const int nb = it % NBAR, n_in = ke - kt < SS ? ke - kt : SS;
              if (__shfl_sync(0xffffffffu, *failed, 0)) {
                stop = true;
                break;
              }
              if (!__all_sync(0xffffffffu, mbar_wait(&sh->full[nb], (it / NBAR) & 1, 4, sp.wait_limit_ns))) {
                *failed = 1;
                stop = true;
                break;
              }
              // The MMAs that last read these slots' columns completed before
              // the producer refilled the slots (their empty barrier), and so
              // before the copies this wait saw land.
              tc_fence_after();
              for (int i = 0; i < n_in; i++) {
                const int st = nb * SS + i;
                if constexpr (BS != B_SPLIT2) {  // B arrives unsplit: each gather warp splits a quarter in place
                  constexpr int per = (int)(TL::B_BYTES / 16) / 4;
                  float4* bh = (float4*)(smem + st * TL::STAGE_BYTES + TL::B_OFF);
                  split_tf32(bh + q * per, bh + TL::B_BYTES / 16 + q * per, per, lane);
                }
                float v[32];
                const uint32_t halo = smem_u32(smem + st * TL::STAGE_BYTES + TL::HALO_OFF);
                if constexpr (AS == A_IM2COL_CK)
                  gather_ck_row_split(ga, halo, hb, mk, v);
                else
                  gather_row_split<AS == A_IM2COL_POS_FULL>(ga, halo, tab_base + 64u * m, live, (kt + i) * BK, hb,
                                                            mk, v);
                __syncwarp();
                tmem_store32(a_lanes + 32 * st, v);
                m = m + r16 >= ga.KHW ? m + r16 - ga.KHW : m + r16;
              }
              tmem_wait_st();
              if constexpr (BS != B_SPLIT2) fence_async_shared();  // generic-proxy writes -> the tensor core
              tc_fence_before();
              __syncwarp();
              if (lane == 0 && !(sp.withhold_arrive && it == 0 && leader)) mbar_arrive_rank(&sh->split[nb], 0);
            }
          }
        }
      } else {
        // ---- splitters (both CTAs): splitter w takes every SPLITTERS-th slice,
        // starting with slice w, whichever ring slot it lands in; a gathered A
        // operand is built here from its halo.
        static_assert(SS == 1, "the splitters take single slices");
        const int sw = warp - SPLIT_WARP0;
        int it = 0;
        bool stop = false;
        int rows4[4] = {0, 0, 0, 0}, kind4[4] = {0, 0, 0, 0};
        if constexpr (AS == A_IM2COL_POS) pos_rows<EK == EK_NCHW_POOL>(ga, lane, rows4);
        for (int u = pair; u < units && !stop; u += pairs) {
          int t, kb, ke;
          unit_of(u, tiles, sp, num_k, t, kb, ke);
          const int a_row = (t / n_tiles) * 2 * BM + (int)rank * BM;
          if constexpr (AS == A_IM2COL_CK) ck_rows(ga, a_row, lane, rows4, kind4);
          if constexpr (AS == A_IM2COL_POS_FULL) pos_rows_full<EK == EK_NCHW_POOL>(ga, a_row, s.M, lane, rows4, kind4);
          for (int kt = kb; kt < ke; kt++, it++) {
            if (it % SPLITTERS != sw) continue;
            const int st = it % STAGES;
            if (__shfl_sync(0xffffffffu, *failed, 0)) {
              stop = true;
              break;
            }
            uint8_t* stage = smem + st * TL::STAGE_BYTES;
            // rows of this CTA's A block that the output uses
            const int a_rows = (int)(s.M - a_row < BM ? (s.M - a_row > 0 ? s.M - a_row : 0) : BM);
            if (!mbar_wait(&sh->full[st], (it / STAGES) & 1, 4, sp.wait_limit_ns)) {
              *failed = 1;
              stop = true;
              break;
            }
            if constexpr (AS == A_TMA) {
              split_tf32((float4*)stage, (float4*)(stage + A_BYTES), A_BYTES / 16, lane);
            } else {
              // im2col tile from the halo in the lo plane into the hi plane,
              // then split in place (the lo plane is overwritten only after
              // every lane has read the halo). Rows past M are left as they
              // are: they only reach rows of C that are never stored.
              const float* halo = (const float*)(stage + TL::HALO_OFF);
              uint8_t* lo = HSEP ? stage + A_BYTES : nullptr;  // with its own halo region: split while gathering
              if constexpr (AS == A_IM2COL_POS || AS == A_IM2COL_POS_FULL)
                gather_pos<AS == A_IM2COL_POS_FULL>(ga, stage, lo, halo, a_rows, kt * BK, lane, rows4, kind4);
              else
                gather_ck(ga, stage, lo, halo, a_rows, lane, rows4, kind4);
              if constexpr (!HSEP) {
                __syncwarp();
                split_tf32((float4*)stage, (float4*)(stage + A_BYTES), a_rows * 64 / 16, lane);
              }
            }
            if constexpr (BS != B_SPLIT2)
              split_tf32((float4*)(stage + TL::B_OFF), (float4*)(stage + TL::B_OFF + TL::B_BYTES), TL::B_BYTES / 16,
                         lane);
            fence_async_shared();  // generic-proxy writes -> visible to the tensor core
            if (!(sp.withhold_arrive && it == 0 && leader)) mbar_arrive_rank(&sh->split[st], 0);
          }
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_HIGH));
    // ---- promoters and epilogue (both CTAs): TMEM lanes 32*(warp%4)..+31 are
    // this warp's rows, columns [HC*h, HC*h + HC) its half of the tile.
    // Every decision below is warp-uniform: tcgen05.ld is .sync.aligned.
    const int q = warp & 3, h = (warp - 8) >> 2;
    // (NCAT: this half's columns with B hi at h * TBN, those with B lo HC after)
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (NCAT ? TBN * h : HC * h);
    float* xpose = (float*)(smem + TL::EPI_OFFSET) + (warp - 8) * 32 * EPI_LD;
    int group = 0;
    for (int u = pair; u < units && !__shfl_sync(0xffffffffu, *failed, 0); u += pairs) {
      int t, kb, ke;
      const int sidx = unit_of(u, tiles, sp, num_k, t, kb, ke);
      // a split unit's partial tile in the workspace (row-major 256 x TBN)
      float* part = sidx < 0 ? nullptr
                             : sp.ws + ((int64_t)sidx * (tiles - sp.whole) + (t - sp.whole)) * TL::TILE_ELEMS +
                                   (int64_t)(rank * BM + 32 * q) * TBN + HC * h + lane;
      const int groups = (ke - kb + GROUP - 1) / GROUP;
      const int mt = t / n_tiles, nt = t % n_tiles;
      // The running total starts at +0 and every partial is added with
      // round-to-nearest, like the reference's c = 0; c += a*b.
      float tot[HC];
#pragma unroll
      for (int i = 0; i < HC; i++) tot[i] = 0.0f;
      bool ok = true;
      for (int g = 0; g < groups; g++, group++) {
        const uint32_t buf = (uint32_t)(group & 1);
        if (!__all_sync(0xffffffffu, mbar_wait(&sh->pfull[buf], (group >> 1) & 1, 7, sp.wait_limit_ns))) {
          *failed = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if constexpr (NCAT) {
          static_assert(HC == 32, "one chunk per half");
          float p[32], pl[32];
          tmem_load32(lane_base + buf * ACC, p);
          tmem_load32(lane_base + buf * ACC + HC, pl);
#pragma unroll
          for (int i = 0; i < 32; i++) tot[i] = __fadd_rn(tot[i], __fadd_rn(p[i], pl[i]));
        } else {
#pragma unroll
          for (int j = 0; j < HC / 32; j++) {
            float p[32];
            tmem_load32(lane_base + buf * ACC + 32 * j, p);
#pragma unroll
            for (int i = 0; i < 32; i++) tot[32 * j + i] = __fadd_rn(tot[32 * j + i], p[i]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_rank(&sh->pempty[buf], 0);  // the buffer may be overwritten
      }
      if (!ok) break;
      const int64_t m0 = (int64_t)mt * 2 * BM + rank * BM + 32 * q;
      const int64_t n0 = (int64_t)nt * TBN + HC * h;
      // The implicit-convolution layouts store each lane's own row (lane =
      // row m): for a column, the warp writes 32 consecutive rows, which are
      // 32 consecutive positions of a channel plane (NCHW) or of a transposed
      // weight-gradient row.
      const int64_t m_own = m0 + lane;
      float* nchw_base = nullptr;
      if constexpr (EK == EK_NCHW_POS) {
        if (!part && m_own < s.M) {
          const int64_t L = epi.nchw_L, img = m_own / L;
          nchw_base = epi.out + img * epi.nchw_M * L + (m_own - img * L);
        }
      }
      // Epilogue: 32 x 32 blocks through the per-warp buffer (the switch keeps
      // the register indices static in a loop that is not unrolled).
#pragma unroll 1
      for (int j = 0; j < HC / 32; j++) {
        switch (j) {
          case 0: xpose_chunk<0>(xpose, tot, lane); break;
          case 1: xpose_chunk<1>(xpose, tot, lane); break;
          case 2: xpose_chunk<2>(xpose, tot, lane); break;
          case 3: xpose_chunk<3>(xpose, tot, lane); break;
        }
        __syncwarp();
        if (part) {
#pragma unroll 4
          for (int r = 0; r < 32; r++) part[r * TBN + 32 * j] = xpose[r * EPI_LD + lane];
        } else if constexpr (EK == EK_NCHW_POS) {
          // the block's 32 biases, one per lane, broadcast by shuffles (a
          // load per column would wait on memory before every store)
          const int64_t nl = n0 + 32 * j + lane;
          const float my_bias = epi.bias && nl < s.N ? __ldg(epi.bias + nl) : 0.0f;
          const int64_t L = epi.nchw_L;
          const bool relu = epi.act == GT_ACT_RELU;
          float* col = nchw_base ? nchw_base + (n0 + 32 * j) * L : nullptr;  // NULL: this lane's row is past M
#pragma unroll 8
          for (int i = 0; i < 32; i++) {
            float v = xpose[lane * EPI_LD + i];
            const float b = __shfl_sync(0xffffffffu, my_bias, i);  // every lane takes part
            if (col && n0 + 32 * j + i < s.N) {
              if (epi.bias) v = __fadd_rn(v, b);
              if (relu) v = go_max(v, 0.0f);
              col[i * L] = v;
            }
          }
        } else if constexpr (EK == EK_NCHW_POOL) {
          // bias, ReLU, then each window's first maximum in offset order
          // (v0 = (0,0), v1 = (0,1), v2 = (1,0), v3 = (1,1): MaxPool2d's
          // v > best rule). Lane 4 w' + k takes channel i0 + k of the warp's
          // window w' (rows 4 w' .. 4 w' + 3 of this warp's buffer; the four
          // reads of a group are conflict-free), so every lane pools and
          // stores.
          const int64_t nl = n0 + 32 * j + lane;
          const float my_bias = epi.bias && nl < s.N ? __ldg(epi.bias + nl) : 0.0f;
          const bool relu = epi.act == GT_ACT_RELU;
          const int64_t P4 = epi.nchw_L / 4;
          const int k = lane & 3, row0 = lane & ~3;
          // lanes 4 w' .. 4 w' + 3 hold window 8 q + w' of the CTA's 32. M is
          // window-major (row 4 w + k of an image's L rows = offset k of its
          // pooled position w), so the window's first row p gives the pooled
          // output: image p / L, position (p % L) / 4; channel c's goes to
          // pool_base + c * P4 (-1: past M).
          int64_t pool_base = -1;
          {
            const int64_t p = (m0 - 32 * q) + 4 * ((32 * q + lane) >> 2);
            if (p < s.M) {
              const int64_t img = p / epi.nchw_L;
              pool_base = img * epi.nchw_M * P4 + (p - img * epi.nchw_L) / 4;
            }
          }
#pragma unroll 1
          for (int i0 = 0; i0 < 32; i0 += 4) {
            const float b = __shfl_sync(0xffffffffu, my_bias, i0 + k);
            float v[4];
#pragma unroll
            for (int p = 0; p < 4; p++) {
              v[p] = xpose[(row0 + p) * EPI_LD + i0 + k];
              if (epi.bias) v[p] = __fadd_rn(v[p], b);
              if (relu) v[p] = go_max(v[p], 0.0f);
            }
            const int64_t c = n0 + 32 * j + i0 + k;
            if (pool_base >= 0 && c < s.N) {
              float best = v[0];
              int kb = 0;
              if (v[1] > best) best = v[1], kb = 1;
              if (v[2] > best) best = v[2], kb = 2;
              if (v[3] > best) best = v[3], kb = 3;
              epi.out[pool_base + c * P4] = best;
              epi.pool_idx[pool_base + c * P4] = (uint8_t)kb;
            }
          }
        } else if constexpr (EK == EK_COLMAJOR) {
          if (m_own < s.M) {
#pragma unroll 4
            for (int i = 0; i < 32; i++) {
              const int64_t n = n0 + 32 * j + i;
              if (n < s.N) {
                const float v = xpose[lane * EPI_LD + i];
                if (m_own == epi.rowsum_m) {
                  if (epi.rowsum_out) epi.rowsum_out[n] = v;
                } else {
                  epi.out[n * epi.ldc + m_own] = v;
                }
              }
            }
          }
        } else {
          epilogue_block<EK>(epi, s, xpose, lane, m0, n0 + 32 * j + lane);
        }
        __syncwarp();
      }
    }
  }

  tc_fence_before();
  __syncwarp();
  __syncthreads();
  cluster_sync();  // no TMEM access remains anywhere in the pair
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TL::TMEM_COLS));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 2-D fp32 tensor map over `outer` rows of `inner` contiguous elements with a
// pitch of `ld` elements; zero fill outside. K-major operands: box 16 x
// box_rows with the 64-byte swizzle; M/N-major: box 32 x 16 with the
// 128-byte swizzle of 32-byte atoms.
static char* make_map(gt_ctx* ctx, CUtensorMap* map, const float* base, int64_t inner, int64_t outer, int64_t ld,
                      bool mn_major, int box_rows = BM) {
  auto encode = (EncodeTiledFn)ctx->encode_tiled;
  if (!encode) return errorf("gemm_tc: cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {mn_major ? 32u : (cuuint32_t)BK, mn_major ? (cuuint32_t)BK : (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                      mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_64B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return errorf("gemm_tc: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return nullptr;
}

// 3-D fp32 tensor map over an (images, channels, L) tensor (dy of a
// convolution, NCHW with the plane flattened): dims {L, channels, images},
// box {16 positions, box_rows channels, 1 image}, the K-major 64-byte swizzle.
// A K-slice of 16 positions is one box when L % 16 == 0.
static char* make_map3(gt_ctx* ctx, CUtensorMap* map, const float* base, int64_t L, int64_t chans, int64_t images,
                       int box_rows) {
  auto encode = (EncodeTiledFn)ctx->encode_tiled;
  if (!encode) return errorf("gemm_tc: cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)L, (cuuint64_t)chans, (cuuint64_t)images};
  cuuint64_t strides[2] = {(cuuint64_t)L * 4, (cuuint64_t)(L * chans) * 4};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return errorf("gemm_tc: cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return nullptr;
}

// 4-D fp32 tensor map over an NCHW tensor, dims {W, H, C, N}, with the halo
// box of a gathered operand (no swizzle: the splitters index it directly);
// zero fill outside the tensor is the convolution's padding.
static char* make_halo_map(gt_ctx* ctx, CUtensorMap* map, const float* base, const gt_geom& g, const Gather& ga) {
  auto encode = (EncodeTiledFn)ctx->encode_tiled;
  if (!encode) return errorf("gemm_tc: cuTensorMapEncodeTiled is unavailable");
  if (ga.full) {  // whole planes: dims {H * W, C, N}
    cuuint64_t dims3[3] = {(cuuint64_t)(g.H * g.W), (cuuint64_t)g.C, (cuuint64_t)g.N};
    cuuint64_t strides3[2] = {(cuuint64_t)(g.H * g.W) * 4, (cuuint64_t)(g.C * g.H * g.W) * 4};
    cuuint32_t box3[3] = {(cuuint32_t)(g.H * g.W), (cuuint32_t)ga.box_c, (cuuint32_t)ga.box_n};
    cuuint32_t estr3[3] = {1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims3, strides3, box3, estr3,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return errorf("gemm_tc: cuTensorMapEncodeTiled (planes) failed (%d)", (int)r);
    return nullptr;
  }
  cuuint64_t dims[4] = {(cuuint64_t)g.W, (cuuint64_t)g.H, (cuuint64_t)g.C, (cuuint64_t)g.N};
  cuuint64_t strides[3] = {(cuuint64_t)g.W * 4, (cuuint64_t)(g.H * g.W) * 4, (cuuint64_t)(g.C * g.H * g.W) * 4};
  cuuint32_t box[4] = {(cuuint32_t)ga.box_w, (cuuint32_t)ga.box_h, (cuuint32_t)ga.box_c, (cuuint32_t)ga.box_n};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return errorf("gemm_tc: cuTensorMapEncodeTiled (halo) failed (%d)", (int)r);
  return nullptr;
}

// SM pairs a GEMM may occupy: all of them, less the SMs reserved for kernels
// that run beside it (a collective on another stream).
static int64_t pairs_available(const gt_ctx* ctx) {
  const int64_t free_sms = (int64_t)ctx->sm_count - ctx->gemm_sm_reserve;
  return free_sms >= 2 ? free_sms / 2 : 1;
}

template <bool A_MN, bool B_MN, int EK, int TBN = BN, int AS = A_TMA, int BS = B_TMA2>
static char* launch_kernel(gt_ctx* ctx, const GemmShape& s, const CUtensorMap& ta, const CUtensorMap& tb,
                           const Epi<float>& epi, const SplitPlan& sp, const Gather& ga) {
  auto kern = gemm_tf32x3_pair_kernel<A_MN, B_MN, EK, TBN, AS, BS>;
  using TL = LayoutOf<TBN, AS>;
  static bool configured[64] = {};
  if (ctx->device < 0 || ctx->device >= 64 || !configured[ctx->device]) {
    GT_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TL::SMEM_BYTES));
    if (ctx->device >= 0 && ctx->device < 64) configured[ctx->device] = true;
  }
  const int64_t tiles = ceil_div(s.M, 2 * BM) * ceil_div(s.N, TBN);
  const int64_t units = sp.whole + (tiles - sp.whole) * sp.splits;
  const int64_t avail = pairs_available(ctx);
  const int64_t pairs = units < avail ? units : avail;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = TL::SMEM_BYTES;
  cfg.stream = ctx->stream;
  GT_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, s, epi, sp, ga));
  GT_LAUNCH_CHECK();
  return nullptr;
}

template <bool A_MN, bool B_MN, int EK>
static char* launch(gt_ctx* ctx, const GemmShape& s, const float* A, const float* B, const Epi<float>& epi,
                    const SplitPlan& sp) {
  CUtensorMap ta, tb;
  if (A_MN)
    GT_TRY(make_map(ctx, &ta, A, s.M, s.K, s.lda, true));
  else
    GT_TRY(make_map(ctx, &ta, A, s.K, s.M, s.lda, false));
  if (B_MN)
    GT_TRY(make_map(ctx, &tb, B, s.N, s.K, s.ldb, true));
  else
    GT_TRY(make_map(ctx, &tb, B, s.K, s.N, s.ldb, false));
  return launch_kernel<A_MN, B_MN, EK>(ctx, s, ta, tb, epi, sp, Gather{});
}

template <int EK>
static char* launch_layout(gt_ctx* ctx, const GemmShape& s, const float* A, const float* B, const Epi<float>& epi,
                           bool a_mn, bool b_mn, const SplitPlan& sp) {
  if constexpr (EK == EK_MASKBITS) {  // only the dX layout (dy row-major, W as N/K-major) is compiled
    if (!a_mn && b_mn) return launch<false, true, EK>(ctx, s, A, B, epi, sp);
    return launch_layout<EK_GENERIC>(ctx, s, A, B, epi, a_mn, b_mn, sp);
  } else {
    if (!a_mn && !b_mn) return launch<false, false, EK>(ctx, s, A, B, epi, sp);
    if (!a_mn && b_mn) return launch<false, true, EK>(ctx, s, A, B, epi, sp);
    if (a_mn && !b_mn) return launch<true, false, EK>(ctx, s, A, B, epi, sp);
    return launch<true, true, EK>(ctx, s, A, B, epi, sp);
  }
}

static char* launch_kind(gt_ctx* ctx, const GemmShape& s, const float* A, const float* B, const Epi<float>& epi,
                         bool a_mn, bool b_mn, const SplitPlan& sp) {
  switch (epi_kind(epi, s.N)) {
    case -1: return errorf("gemm_tc: a ReLU bit mask needs a row-major bias / ReLU epilogue");
    case -2: return errorf("gemm_tc: a convolution layout with an unsupported epilogue");
    case EK_MASKBITS: return launch_layout<EK_MASKBITS>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    case EK_PLAIN: return launch_layout<EK_PLAIN>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    case EK_BIAS_RELU: return launch_layout<EK_BIAS_RELU>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    case EK_MASK: return launch_layout<EK_MASK>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    case EK_CONV: return launch_layout<EK_CONV>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    case EK_NCHW_POS:
    case EK_NCHW_POOL:
    case EK_COLMAJOR: return errorf("gemm_tc: the implicit convolution layouts have their own launchers");
    default: return launch_layout<EK_GENERIC>(ctx, s, A, B, epi, a_mn, b_mn, sp);
  }
}

// C of the split tiles = epilogue(sum of their partials), the partials added
// in split order, so the result does not depend on which unit finished first.
template <int TBN>
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, SplitPlan sp, int tiles, int n_tiles, int64_t M,
                                     int64_t N, Epi<float> epi) {
  constexpr int64_t TE = Tile<TBN>::TILE_ELEMS;
  const int rest = tiles - sp.whole;
  const int64_t total = (int64_t)rest * TE;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / TE);
    const int64_t e = i - (int64_t)r * TE;
    const int t = sp.whole + r;
    const int64_t m = (int64_t)(t / n_tiles) * 2 * BM + e / TBN, n = (int64_t)(t % n_tiles) * TBN + e % TBN;
    if (m >= M || n >= N) continue;
    float acc = ws[i];
    for (int k = 1; k < sp.splits; k++) acc = __fadd_rn(acc, ws[(int64_t)k * total + i]);
    epi.store(m, n, acc);
  }
}

// The split tiles of a pooled implicit convolution (EK_NCHW_POOL): a thread
// finishes the four rows of one 2 x 2 window (rows 4 w .. 4 w + 3 of a CTA,
// Gather::pool2) for one channel, each summed in split order as
// splitk_reduce_kernel sums it, and stores the window's first maximum and its
// offset, as the kernel's own pooled epilogue does for whole tiles.
template <int TBN>
__global__ void splitk_reduce_pool_kernel(const float* __restrict__ ws, SplitPlan sp, int tiles, int n_tiles,
                                          int64_t M, int64_t N, Epi<float> epi) {
  constexpr int64_t TE = Tile<TBN>::TILE_ELEMS;
  const int rest = tiles - sp.whole;
  const int64_t total = (int64_t)rest * TE, work = (int64_t)rest * 2 * (BM / 4) * TBN;
  const int64_t L = epi.nchw_L, P4 = L / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < work; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / (2 * (BM / 4) * TBN));
    const int64_t e = i - (int64_t)r * 2 * (BM / 4) * TBN;
    const int wg = (int)(e / TBN), cl = (int)(e - (int64_t)wg * TBN);
    const int t = sp.whole + r;
    const int64_t n = (int64_t)(t % n_tiles) * TBN + cl;
    if (n >= N) continue;
    const int rank = wg / (BM / 4), w = wg - rank * (BM / 4);
    const int64_t m_tl = (int64_t)(t / n_tiles) * 2 * BM + rank * BM + 4 * w;  // the window's first row (window-major)
    if (m_tl >= M) continue;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int64_t at = (int64_t)r * TE + (int64_t)(rank * BM + 4 * w + k) * TBN + cl;
      float acc = ws[at];
      for (int s = 1; s < sp.splits; s++) acc = __fadd_rn(acc, ws[(int64_t)s * total + at]);
      v[k] = epi.finish(m_tl, n, acc);
    }
    float best = v[0];
    int kb = 0;
    if (v[1] > best) best = v[1], kb = 1;
    if (v[2] > best) best = v[2], kb = 2;
    if (v[3] > best) best = v[3], kb = 3;
    const int64_t img = m_tl / L;
    const int64_t o = (img * epi.nchw_M + n) * P4 + (m_tl - img * L) / 4;
    epi.out[o] = best;
    epi.pool_idx[o] = (uint8_t)kb;
  }
}

// The same with column partial sums (Epi::colsum_ws): a thread finishes one
// column of 32 rows of a split tile and adds the finished values in row order.
template <int TBN>
__global__ void splitk_reduce_colsum_kernel(const float* __restrict__ ws, SplitPlan sp, int tiles, int n_tiles,
                                            int64_t M, int64_t N, Epi<float> epi) {
  constexpr int64_t TE = Tile<TBN>::TILE_ELEMS;
  const int rest = tiles - sp.whole;
  const int64_t total = (int64_t)rest * TE;
  const int64_t units = total / 32;  // (tile, 32-row block, column)
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(u / (TE / 32));
    const int64_t v = u - (int64_t)r * (TE / 32);
    const int rb = (int)(v / TBN), c = (int)(v % TBN);
    const int t = sp.whole + r;
    const int64_t m0 = (int64_t)(t / n_tiles) * 2 * BM + 32 * rb, n = (int64_t)(t % n_tiles) * TBN + c;
    if (m0 >= M || n >= N) continue;
    float cs = 0.0f;
    for (int j = 0; j < 32 && m0 + j < M; j++) {
      const int64_t i = (int64_t)r * TE + (int64_t)(32 * rb + j) * TBN + c;
      float acc = ws[i];
      for (int k = 1; k < sp.splits; k++) acc = __fadd_rn(acc, ws[(int64_t)k * total + i]);
      const float y = epi.finish(m0 + j, n, acc);
      epi.put(m0 + j, n, y);
      cs = __fadd_rn(cs, y);
    }
    epi.colsum_ws[(m0 >> 5) * epi.ldcs + n] = cs;
  }
}

// The split tiles of a GEMM whose epilogue also writes the ReLU bit mask: a
// 256-thread block per 32 x 32 block of a split tile; thread (ty, tx) adds the
// partials of rows ty, ty + 8, ty + 16, ty + 24 of column tx in split order
// (coalesced along the columns), stores the finished values, and leaves their
// signs in shared memory, from which warp 0 builds the column words.
__global__ void __launch_bounds__(256) splitk_reduce_bits_kernel(const float* __restrict__ ws, SplitPlan sp,
                                                                 int tiles, int n_tiles, int64_t M, int64_t N,
                                                                 Epi<float> epi) {
  __shared__ uint32_t pos[32][33];
  const int rest = tiles - sp.whole;
  const int64_t total = (int64_t)rest * TILE_ELEMS;
  const int64_t blocks = total / 1024;  // (tile, 32-row block, 32-column block)
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int64_t u = blockIdx.x; u < blocks; u += gridDim.x) {
    const int r = (int)(u / (TILE_ELEMS / 1024));
    const int v = (int)(u - (int64_t)r * (TILE_ELEMS / 1024));
    const int rb = v / (BN / 32), cb = v % (BN / 32);
    const int t = sp.whole + r;
    const int64_t m0 = (int64_t)(t / n_tiles) * 2 * BM + 32 * rb, n = (int64_t)(t % n_tiles) * BN + 32 * cb + tx;
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int j = ty + 8 * q;
      uint32_t bit = 0;
      if (m0 + j < M && n < N) {
        const int64_t i = (int64_t)r * TILE_ELEMS + (int64_t)(32 * rb + j) * BN + 32 * cb + tx;
        float acc = ws[i];
#pragma unroll 4
        for (int k = 1; k < sp.splits; k++) acc = __fadd_rn(acc, ws[(int64_t)k * total + i]);
        const float y = epi.finish(m0 + j, n, acc);
        epi.put(m0 + j, n, y);
        bit = y > 0.0f;
      }
      pos[j][tx] = bit;
    }
    __syncthreads();
    if (ty == 0 && m0 < M && n < N) {
      uint32_t w = 0;
#pragma unroll
      for (int j = 0; j < 32; j++) w |= pos[j][tx] << j;
      epi.bits_out[(m0 >> 5) * epi.ldw + n] = w;
    }
    __syncthreads();
  }
}

// The split plan of a GEMM, from a cost model in units of one K-slice of MMA
// on a pair (~0.54 us): rounds x (slices per unit + a fixed per-unit
// overhead), plus the partials' trip through memory at ~5 TB/s. Candidates:
// no split; every tile split S ways (too few tiles for the SM pairs); or only
// the tiles of a mostly empty last round split S ways (wave quantisation).
static int g_force_splits = 0;
static uint64_t g_wait_limit_ns = kTimeoutNs;  // gt_debug_set_tc_wait_limit_us
static int g_withhold_next = 0;               // gt_debug_tc_withhold_arrive

static SplitPlan choose_plan(int64_t tiles, int64_t pairs, int64_t num_k, int64_t tile_elems = TILE_ELEMS) {
  SplitPlan best;
  best.whole = (int)tiles;
  if (g_force_splits > 1) {
    best.whole = 0;
    best.splits = (int)std::min<int64_t>(g_force_splits, std::max<int64_t>(num_k, 1));
    return best;
  }
  constexpr double kUnitOverhead = 40.0;
  auto reduce_cost = [&](int64_t split_tiles, int S) {
    // a slice's MMA time scales with the tile width; so does the partials' traffic
    return (S + 1) * (double)split_tiles * TILE_ELEMS * 4.0 / 5e6 / 0.54;
  };
  const double base = std::ceil((double)tiles / pairs) * (num_k + kUnitOverhead);
  double best_cost = base;
  for (int S = 2; S <= 64 && num_k / S >= 2 * GROUP; S++) {
    // every tile split (the workspace holds S partial tiles per tile: at most 1 GB)
    double c = (double)S * tiles * tile_elems * 4 > (double)(1ull << 30)
                   ? INFINITY
                   : std::ceil((double)(tiles * S) / pairs) * (std::ceil((double)num_k / S) + kUnitOverhead) +
                         reduce_cost(tiles, S);
    if (c < best_cost) {
      best_cost = c;
      best.whole = 0;
      best.splits = S;
    }
    // only the last round's tiles split
    const int64_t full = tiles / pairs * pairs, rest = tiles - full;
    if (full > 0 && rest > 0 && rest * S <= pairs) {
      c = (double)(tiles / pairs) * (num_k + kUnitOverhead) + std::ceil((double)num_k / S) + kUnitOverhead +
          reduce_cost(rest, S);
      if (c < best_cost) {
        best_cost = c;
        best.whole = (int)full;
        best.splits = S;
      }
    }
  }
  if (best_cost > 0.93 * base) {  // measured: smaller gains do not pay
    best.whole = (int)tiles;
    best.splits = 1;
  }
  return best;
}

// Runs a tcgen05 GEMM of `tiles` tiles (`n_tiles` per row of tiles) with the
// split plan its shape calls for: fire(plan) launches the main kernel; split
// units leave partial tiles in a pool workspace that a second kernel sums in
// split order and finishes with the epilogue.
template <int TBN, typename Fire>
static char* run_planned(gt_ctx* ctx, const GemmShape& s, const Epi<float>& epi, int64_t tiles, int64_t n_tiles,
                         Fire&& fire, const Gather* ga = nullptr) {
  constexpr int64_t TE = Tile<TBN>::TILE_ELEMS;
  SplitPlan sp = choose_plan(tiles, pairs_available(ctx), ceil_div(s.K, BK), TE);
  sp.wait_limit_ns = g_wait_limit_ns;
  sp.withhold_arrive = g_withhold_next;
  g_withhold_next = 0;
  if (sp.splits <= 1) return fire(sp);
  const int64_t rest = tiles - sp.whole;
  void* ws = nullptr;
  GT_TRY(scratch(ctx, (size_t)sp.splits * rest * TE * sizeof(float), &ws));
  sp.ws = (float*)ws;
  char* err = fire(sp);
  if (!err) {
    if (epi.pool_idx)  // pooled implicit convolution (ga set by its launcher)
      splitk_reduce_pool_kernel<TBN><<<grid_for(ctx, rest * TE / 4, 256), 256, 0, ctx->stream>>>(
          sp.ws, sp, (int)tiles, (int)n_tiles, s.M, s.N, epi);
    else if (epi.bits_out)
      splitk_reduce_bits_kernel<<<(unsigned)std::min<int64_t>(rest * TE / 1024, (int64_t)ctx->sm_count * 8), 256, 0,
                                  ctx->stream>>>(
          sp.ws, sp, (int)tiles, (int)n_tiles, s.M, s.N, epi);
    else if (epi.colsum_ws)
      splitk_reduce_colsum_kernel<TBN><<<grid_for(ctx, rest * TE / 32, 256), 256, 0, ctx->stream>>>(
          sp.ws, sp, (int)tiles, (int)n_tiles, s.M, s.N, epi);
    else
      splitk_reduce_kernel<TBN><<<grid_for(ctx, rest * TE, 256), 256, 0, ctx->stream>>>(sp.ws, sp, (int)tiles,
                                                                                        (int)n_tiles, s.M, s.N, epi);
    count_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) err = cuda_error(e, "splitk_reduce_kernel launch", __FILE__, __LINE__);
  }
  release(ctx, ws);
  return err;
}

template <int TBN>
static char* conv_fwd_launch(gt_ctx* ctx, const GemmShape& s, const CUtensorMap& ta, const CUtensorMap& tb,
                             const Epi<float>& e, const Gather& ga) {
  const int64_t n_tiles = ceil_div(s.N, TBN), tiles = ceil_div(s.M, 2 * BM) * n_tiles;
  return run_planned<TBN>(ctx, s, e, tiles, n_tiles, [&](const SplitPlan& sp) {
    return ga.full ? launch_kernel<false, false, EK_NCHW_POS, TBN, A_IM2COL_POS_FULL, B_SPLIT2>(ctx, s, ta, tb, e, sp, ga)
                   : launch_kernel<false, false, EK_NCHW_POS, TBN, A_IM2COL_POS, B_SPLIT2>(ctx, s, ta, tb, e, sp, ga);
  });
}

// The forward with 2 x 2 pooling in the epilogue; split tiles are pooled by
// splitk_reduce_pool_kernel. The split plan is the unpooled forward's, so the
// pooled values are those of conv_fwd_launch followed by pooling, bit for bit.
template <int TBN>
static char* conv_fwd_pool_launch(gt_ctx* ctx, const GemmShape& s, const CUtensorMap& ta, const CUtensorMap& tb,
                                  const Epi<float>& e, const Gather& ga) {
  const int64_t n_tiles = ceil_div(s.N, TBN), tiles = ceil_div(s.M, 2 * BM) * n_tiles;
  return run_planned<TBN>(
      ctx, s, e, tiles, n_tiles,
      [&](const SplitPlan& sp) {
        return ga.full
                   ? launch_kernel<false, false, EK_NCHW_POOL, TBN, A_IM2COL_POS_FULL, B_SPLIT2>(ctx, s, ta, tb, e, sp, ga)
                   : launch_kernel<false, false, EK_NCHW_POOL, TBN, A_IM2COL_POS, B_SPLIT2>(ctx, s, ta, tb, e, sp, ga);
      },
      &ga);
}

template <int TBN>
static char* conv_wgrad_launch(gt_ctx* ctx, const GemmShape& s, const CUtensorMap& ta, const CUtensorMap& tb,
                               const Epi<float>& e, const Gather& ga) {
  const int64_t n_tiles = ceil_div(s.N, TBN), tiles = ceil_div(s.M, 2 * BM) * n_tiles;
  return run_planned<TBN>(ctx, s, e, tiles, n_tiles, [&](const SplitPlan& sp) {
    return launch_kernel<false, false, EK_COLMAJOR, TBN, A_IM2COL_CK, B_TMA3>(ctx, s, ta, tb, e, sp, ga);
  });
}

// The halo geometry shared by both orientations (stride 1 only); false if
// the geometry does not fit the implicit path.
static bool halo_common(const gt_geom& g, Gather& ga) {
  if (g.stride != 1 || g.pad < 0 || g.pad > 64 || g.W % 4 || g.KH > 64 || g.KW > 64) return false;
  ga.C = (int)g.C, ga.H = (int)g.H, ga.W = (int)g.W, ga.KH = (int)g.KH, ga.KW = (int)g.KW, ga.OW = (int)g.OW;
  ga.pad = (int)g.pad, ga.L = (int)(g.OH * g.OW), ga.KHW = (int)(g.KH * g.KW), ga.CKK = (int)(g.C * g.KH * g.KW);
  ga.rp = (ga.pad + 3) / 4 * 4;
  return true;
}

// Most channels that `span` consecutive patch entries starting at a multiple
// of `span` touch (the pattern repeats every lcm(span, KHW) entries).
static int channels_spanned(int span, int khw, int C) {
  int most = 1;
  for (int k0 = 0; k0 < span * khw; k0 += span) most = std::max(most, (k0 + span - 1) / khw - k0 / khw + 1);
  return std::min(most, C);
}

static bool halo_fits(Gather& ga) {
  const int64_t floats = (int64_t)ga.box_w * ga.box_h * ga.box_c * ga.box_n;
  if (ga.box_w > 256 || ga.box_h > 256 || ga.box_c > 256 || ga.box_n > 256 || floats * 4 > A_BYTES) return false;
  ga.halo_bytes = (uint32_t)(floats * 4);
  return true;
}

// A_IM2COL_POS: a CTA's 128 positions are whole output rows of one image
// (L % 128 == 0 and 128 % OW == 0) or whole images (128 % L == 0), and the
// halo box covers just them; otherwise (Gather::full) the box holds the whole
// padded images that any 128 consecutive positions touch, if that fits.
static bool halo_pos(const gt_geom& g, Gather& ga) {
  if (!halo_common(g, ga) || ga.KHW > 64) return false;  // the tap table holds 64 taps
  const int64_t L = g.OH * g.OW;
  if (L % 128 == 0 && 128 % g.OW == 0) {
    ga.bh = (int)(128 / g.OW), ga.box_n = 1;
  } else if (L < 128 && 128 % L == 0) {
    ga.bh = (int)g.OH, ga.box_n = (int)(128 / L);
  } else {
    return false;
  }
  ga.rows_pi = ga.bh * ga.OW;
  ga.box_w = (int)((g.OW + g.KW - 1 + ga.rp - g.pad + 3) / 4 * 4);
  ga.box_h = ga.bh + ga.KH - 1;
  ga.box_c = channels_spanned(BK, ga.KHW, ga.C);
  return halo_fits(ga);
}

// A_IM2COL_CK: a slice's 16 positions must form whole rows of 16 columns
// (OW % 16 == 0) or whole rows of one image (16 % OW == 0, L % 16 == 0).
static bool halo_ck(const gt_geom& g, Gather& ga) {
  if (!halo_common(g, ga)) return false;
  if (g.OW % 16 == 0) {
    ga.w16 = 16, ga.r16 = 1;
  } else if (16 % g.OW == 0 && (g.OH * g.OW) % 16 == 0) {
    ga.w16 = (int)g.OW, ga.r16 = (int)(16 / g.OW);
  } else {
    return false;
  }
  ga.box_w = (ga.w16 + ga.KW - 1 + ga.rp - ga.pad + 3) / 4 * 4;
  ga.box_h = ga.r16 + ga.KH - 1;
  ga.box_c = channels_spanned(BM, ga.KHW, ga.C);
  ga.box_n = 1;
  return halo_fits(ga);
}

// A_IM2COL_POS_FULL: whole image planes of H x W <= 256 elements (a
// multiple of 4, so that each plane starts 16-byte aligned), loaded by a 3-D
// map over (H * W, C, N) for any 128 consecutive positions, if they fit.
static bool halo_pos_full(const gt_geom& g, Gather& ga) {
  const int64_t plane = g.H * g.W, L = g.OH * g.OW;
  if (g.stride != 1 || plane > 256 || plane % 4 || g.KH * g.KW > 32 || g.pad > 64 || L < 1) return false;  // 32 mask bits
  ga.C = (int)g.C, ga.H = (int)g.H, ga.W = (int)g.W, ga.KH = (int)g.KH, ga.KW = (int)g.KW, ga.OW = (int)g.OW;
  ga.pad = (int)g.pad, ga.L = (int)L, ga.KHW = (int)(g.KH * g.KW), ga.CKK = (int)(g.C * g.KH * g.KW);
  ga.rp = 0, ga.full = 1;
  ga.bh = (int)g.OH, ga.rows_pi = (int)L;
  ga.box_w = (int)g.W, ga.box_h = (int)g.H;
  ga.box_c = channels_spanned(BK, ga.KHW, ga.C);
  ga.box_n = (int)(1 + (127 + L - 1) / L);
  return halo_fits(ga);
}

static bool fits32(const gt_geom& g, int64_t chans_out) {
  const int64_t lim = INT32_MAX / 2;
  return g.N * g.C * g.H * g.W < lim && g.N * g.OH * g.OW < lim && g.C * g.KH * g.KW < lim &&
         g.N * chans_out * g.OH * g.OW < lim && g.H < lim / 4 && g.W < lim / 4 && g.stride < 65536 &&
         g.pad < 65536 && g.KH < 65536 && g.KW < 65536;
}

}  // namespace tc

void set_gemm_splits(int splits) { tc::g_force_splits = splits; }
void set_tc_wait_limit_us(int64_t us) { tc::g_wait_limit_ns = us > 0 ? (uint64_t)us * 1000ull : tc::kTimeoutNs; }
void tc_withhold_next_arrive() { tc::g_withhold_next = 1; }

// Reports (and clears) a timed-out pipeline wait of an earlier tcgen05 GEMM.
char* tc_check_errors() {
  int e = 0;
  GT_CUDA(cudaMemcpyFromSymbol(&e, g_tc_error, sizeof e));
  if (e) {
    int zero = 0;
    cudaMemcpyToSymbol(g_tc_error, &zero, sizeof zero);
    return errorf("tcgen05 GEMM: a pipeline wait timed out (site %d); results are invalid", e);
  }
  return nullptr;
}

bool tc_writes_colsums(const Epi<float>& epi, int64_t n_cols) {
  const int k = tc::epi_kind(epi, n_cols);
  return k == tc::EK_PLAIN || k == tc::EK_MASK || k == tc::EK_MASKBITS;
}

char* gemm_tc_f32(gt_ctx* ctx, const GemmShape& s, const float* A, const float* B, const Epi<float>& epi,
                  bool* done) {
  *done = false;
  // TMA needs 16-byte aligned bases and row pitches; tiny problems stay on SIMT.
  if (((uintptr_t)A & 15) || ((uintptr_t)B & 15) || (s.lda & 3) || (s.ldb & 3)) return nullptr;
  if (s.M < 1 || s.N < 1 || s.K < 1 || s.M > INT32_MAX / 2 || s.N > INT32_MAX / 2 || s.K > INT32_MAX / 2)
    return nullptr;
  if (ctx->sm_count < 2) return nullptr;
  if (gemm_path() != 2 && s.M * s.N * s.K < (int64_t)1 << 21) return nullptr;
  if (epi.pos_major || epi.col_major) return nullptr;  // the implicit-convolution layouts have their own launchers
  const bool a_mn = s.trans_a, b_mn = !s.trans_b;
  const int64_t n_tiles = ceil_div(s.N, tc::BN), tiles = ceil_div(s.M, 2 * tc::BM) * n_tiles;
  char* err = tc::run_planned<tc::BN>(ctx, s, epi, tiles, n_tiles, [&](const tc::SplitPlan& sp) {
    return tc::launch_kind(ctx, s, A, B, epi, a_mn, b_mn, sp);
  });
  if (!err) *done = true;
  return err;
}

char* conv_fwd_tc(gt_ctx* ctx, const float* x, const float* ws, int64_t w_pitch, const float* bias, float* y,
                  const gt_geom& g, int64_t O, int act, bool* done, uint8_t* pool_idx) {
  *done = false;
  const int64_t L = g.OH * g.OW, P = g.N * L, CKK = g.C * g.KH * g.KW;
  if (P < 1 || O < 1 || CKK < 1 || ctx->sm_count < 2 || !tc::fits32(g, O)) return nullptr;
  if (((uintptr_t)ws & 15) || (w_pitch & 3) || w_pitch < CKK || (act != GT_ACT_NONE && act != GT_ACT_RELU))
    return nullptr;
  // C (P, O) = cols (P, CKK) @ w (O, CKK)^T: A gathered, B(k, n) = w[n * w_pitch + k].
  GemmShape s{P, O, CKK, false, true, 0, w_pitch};
  tc::Gather ga;
  if ((uintptr_t)x & 15) return nullptr;
  if (!tc::halo_pos(g, ga)) {
    ga = tc::Gather();
    if (!tc::halo_pos_full(g, ga)) return nullptr;
  }
  if (pool_idx) {
    // windows must not straddle CTAs: a CTA's 128 positions are whole row
    // pairs of one image (an even number of rows) or whole images
    if (g.OH % 2 || g.OW % 2 || (!ga.full && ga.box_n == 1 && ga.bh % 2)) return nullptr;
    ga.pool2 = 1;
  }
  ga.b_lo_row = (int)conv_weight_rows(O);
  Epi<float> e;
  e.out = y;
  e.bias = bias;
  e.act = act;
  e.nchw_L = L;
  e.nchw_M = O;
  e.pos_major = true;
  e.pool_idx = pool_idx;
  const int tbn = (int)conv_tile_width(O);
  CUtensorMap ta, tb;
  GT_TRY(tc::make_halo_map(ctx, &ta, x, g, ga));
  GT_TRY(tc::make_map(ctx, &tb, ws, CKK, 2 * ga.b_lo_row, w_pitch, false, tbn / 2));
  char* err = nullptr;
  if (pool_idx)
    err = tbn == 64    ? tc::conv_fwd_pool_launch<64>(ctx, s, ta, tb, e, ga)
          : tbn == 128 ? tc::conv_fwd_pool_launch<128>(ctx, s, ta, tb, e, ga)
                       : tc::conv_fwd_pool_launch<256>(ctx, s, ta, tb, e, ga);
  else
    err = tbn == 64    ? tc::conv_fwd_launch<64>(ctx, s, ta, tb, e, ga)
          : tbn == 128 ? tc::conv_fwd_launch<128>(ctx, s, ta, tb, e, ga)
                       : tc::conv_fwd_launch<256>(ctx, s, ta, tb, e, ga);
  if (!err) *done = true;
  return err;
}

char* conv_wgrad_tc(gt_ctx* ctx, const float* x, const float* dy, float* dw, float* db, const gt_geom& g, int64_t O,
                    bool* done) {
  *done = false;
  const int64_t L = g.OH * g.OW, P = g.N * L, CKK = g.C * g.KH * g.KW;
  if (P < 1 || O < 1 || CKK < 1 || ctx->sm_count < 2 || !tc::fits32(g, O)) return nullptr;
  // A K-slice of 16 positions must lie in one image and start 16-byte aligned.
  if (L % 16 || ((uintptr_t)dy & 15)) return nullptr;
  // C (CKK [+1], O) = cols^T (CKK, P) @ dy (P, O); the extra row of ones in
  // A makes row CKK of C the bias gradient.
  GemmShape s{CKK + (db ? 1 : 0), O, P, true, false, 0, 0};
  tc::Gather ga;
  if (!tc::halo_ck(g, ga) || ((uintptr_t)x & 15)) return nullptr;
  ga.ones_row = db ? (int)CKK : -1;
  Epi<float> e;
  e.out = dw;
  e.ldc = CKK;
  e.col_major = true;
  e.rowsum_out = db;
  e.rowsum_m = db ? CKK : -1;
  const int tbn = (int)conv_tile_width(O);
  CUtensorMap ta, tb;
  GT_TRY(tc::make_halo_map(ctx, &ta, x, g, ga));
  GT_TRY(tc::make_map3(ctx, &tb, dy, L, O, g.N, tbn / 2));
  char* err = tbn == 64    ? tc::conv_wgrad_launch<64>(ctx, s, ta, tb, e, ga)
              : tbn == 128 ? tc::conv_wgrad_launch<128>(ctx, s, ta, tb, e, ga)
                           : tc::conv_wgrad_launch<256>(ctx, s, ta, tb, e, ga);
  if (!err) *done = true;
  return err;
}

}  // namespace gt
