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
//               partial accumulator, commits that free the slot in both CTAs;
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
// Every barrier wait is bounded in time; on expiry the kernel records the
// waiting site in an error word (reported by gt_sync), stops its loops,
// waits (bounded) for its copies and MMAs in flight, frees its tensor memory
// and returns instead of hanging the GPU. No thread returns early, so the
// closing cluster barrier is always reached by every thread.
#include <cuda.h>

#include <algorithm>
#include <cmath>

#include "gemm.cuh"

namespace gt {

__device__ int g_tc_error = 0;

namespace tc {

constexpr int BM = 128;    // A rows per CTA (a pair covers 256)
constexpr int BN = 256;    // C columns per tile
constexpr int BNH = 128;   // B rows per CTA
constexpr int BK = 16;     // K elements per slice
constexpr int STAGES = 6;
constexpr int GROUP = 16;  // K slices per promotion group
constexpr int THREADS = 512;
constexpr int SPLIT_WARP0 = 2;  // warps 2..2+STAGES-1 split; warp 2+j owns slot j
constexpr int PROMOTERS = 256;
constexpr uint32_t A_BYTES = BM * BK * 4;
constexpr uint32_t B_BYTES = BNH * BK * 4;
constexpr uint32_t STAGE_BYTES = 2 * (A_BYTES + B_BYTES);  // A hi, A lo, B hi, B lo
constexpr uint32_t BAR_OFFSET = STAGES * STAGE_BYTES;
constexpr int PROMOTER_WARPS = PROMOTERS / 32;
constexpr int EPI_LD = 33;  // padded row of the per-warp 32 x 32 transpose (conflict-free both ways)
constexpr uint32_t EPI_OFFSET = BAR_OFFSET + 512;
constexpr uint32_t EPI_BYTES = PROMOTER_WARPS * 32 * EPI_LD * 4;
constexpr uint32_t SMEM_BYTES = EPI_OFFSET + EPI_BYTES + 1024;  // + slack for 1024-byte alignment
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t BUF_COLS = 256;  // one partial accumulator: 128 lanes x 256 fp32 columns
// Registers per thread after the split: warps 0-7 (TMA, MMA, splitters) and
// warps 8-15 (promoters). The launch gives every thread 65536 / 512 = 128;
// the split keeps the block's total: 256 * 64 + 256 * 192 = 256 * 128 * 2.
constexpr int REGS_LOW = 64, REGS_HIGH = 192;
static_assert(256 * REGS_LOW + 256 * REGS_HIGH <= THREADS * 128, "register split exceeds the launch's registers");
constexpr uint64_t kTimeoutNs = 2000000000ull;  // default limit, 2 s; a healthy wait takes microseconds

static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

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

// Instruction descriptor for kind::tf32, fp32 accumulate, M = 256 (pair), N = 256.
template <bool A_MN, bool B_MN>
__device__ __forceinline__ uint32_t instr_desc() {
  uint32_t d = 0;
  d |= 1u << 4;                 // D format: F32
  d |= 2u << 7;                 // A format: TF32
  d |= 2u << 10;                // B format: TF32
  d |= (A_MN ? 1u : 0u) << 15;  // A major
  d |= (B_MN ? 1u : 0u) << 16;  // B major
  d |= (uint32_t)(BN >> 3) << 17;
  d |= (uint32_t)((2 * BM) >> 4) << 24;
  return d;
}

__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0),
      "r"(0)
      : "memory");
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

// Rounds to the nearest tf32 value (ties away from zero) on the integer ALU:
// add half a tf32 ulp to the magnitude bits, clear the 13 dropped bits. (The
// cvt instruction for this runs on the narrow XU pipe, which capped the
// splitters at a third of the tensor rate.) Infinities stay infinities; a
// NaN stays NaN or becomes an infinity whose lo part is NaN, so the product
// is NaN either way.
__device__ __forceinline__ float tf32_round(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
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
};

inline int epi_kind(const Epi<float>& e, int64_t n_cols) {
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
  if (EK == EK_PLAIN) {
#pragma unroll 4
    for (int r = 0; r < rows; r++) op[r * epi.ldc] = xpose[r * EPI_LD + lane];
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
    for (int r = 0; r < rows; r++) op[r * epi.ldc] = __fmul_rn(xpose[r * EPI_LD + lane], ((w >> r) & 1u) ? 1.0f : 0.0f);
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
        if (r0 + r < rows) op[(r0 + r) * epi.ldc] = act_bwd(epi.dact, xpose[(r0 + r) * EPI_LD + lane], mask[r]);
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
  uint64_t full[STAGES];   // TMA -> splitters (local)
  uint64_t split[STAGES];  // splitters of both CTAs -> leader's MMA
  uint64_t empty[STAGES];  // MMA -> producers of both CTAs
  uint64_t pfull[2];       // MMA -> promoters of both CTAs: partial buffer b is complete
  uint64_t pempty[2];      // promoter warps of both CTAs -> leader's MMA: buffer b was read
  uint64_t mma_done;       // leader: every MMA issued has completed
  uint32_t tmem_base;
  int failed;
};

template <bool A_MN, bool B_MN, int EK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_tf32x3_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            GemmShape s, Epi<float> epi, SplitPlan sp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  Shared* sh = (Shared*)(smem + BAR_OFFSET);
  volatile int* failed = &sh->failed;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int num_k = (int)((s.K + BK - 1) / BK);
  const int m_tiles = (int)((s.M + 2 * BM - 1) / (2 * BM));
  const int n_tiles = (int)((s.N + BN - 1) / BN);
  const int tiles = m_tiles * n_tiles;
  const int units = sp.whole + (tiles - sp.whole) * sp.splits;
  const int pair = (int)cluster_id(), pairs = (int)num_clusters();

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; i++) {
      mbar_init(&sh->full[i], 1);
      mbar_init(&sh->split[i], 2 * 32);  // one splitter warp per CTA per slice
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
                 "r"(TMEM_COLS));
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
      if (lane == 0) {  // ---- TMA producer (both CTAs)
        int it = 0, issued_to = 0;
        for (int u = pair; u < units && !*failed; u += pairs) {
          int t, kb, ke;
          unit_of(u, tiles, sp, num_k, t, kb, ke);
          const int mt = t / n_tiles, nt = t % n_tiles;
          const int a_row = mt * 2 * BM + (int)rank * BM;
          const int b_row = nt * BN + (int)rank * BNH;
          for (int kt = kb; kt < ke; kt++, it++) {
            const int st = it % STAGES;
            if (!mbar_wait(&sh->empty[st], ((it / STAGES) & 1) ^ 1, 1, sp.wait_limit_ns)) {
              *failed = 1;
              break;
            }
            uint8_t* a_hi = smem + st * STAGE_BYTES;
            uint8_t* b_hi = a_hi + 2 * A_BYTES;
            mbar_expect_tx(&sh->full[st], A_BYTES + B_BYTES);
            const int k0 = kt * BK;
            if (A_MN) {
  #pragma unroll
              for (int j = 0; j < BM / 32; j++) tma_load_2d(a_hi + j * kLboMN, &tmA, &sh->full[st], a_row + 32 * j, k0);
            } else {
              tma_load_2d(a_hi, &tmA, &sh->full[st], k0, a_row);
            }
            if (B_MN) {
  #pragma unroll
              for (int j = 0; j < BNH / 32; j++)
                tma_load_2d(b_hi + j * kLboMN, &tmB, &sh->full[st], b_row + 32 * j, k0);
            } else {
              tma_load_2d(b_hi, &tmB, &sh->full[st], k0, b_row);
            }
            issued_to = it + 1;
          }
        }
        if (*failed) {  // let copies in flight land before the CTA tears down
          for (int i = issued_to > STAGES ? issued_to - STAGES : 0; i < issued_to; i++)
            mbar_wait(&sh->full[i % STAGES], (i / STAGES) & 1, 5, kTimeoutNs);  // copies land in microseconds
        }
      }
    } else if (warp == 1) {
      if (lane == 0 && leader) {  // ---- MMA issuer (leader CTA only)
        const uint32_t idesc = instr_desc<A_MN, B_MN>();
        int it = 0, group = 0;
        bool stop = false;
        for (int u = pair; u < units && !stop; u += pairs) {
          int t, kb, ke;
          unit_of(u, tiles, sp, num_k, t, kb, ke);
          for (int kt = kb; kt < ke; kt++, it++) {
            const bool group_start = (kt - kb) % GROUP == 0;
            const uint32_t buf = (uint32_t)(group & 1);
            if (group_start) {  // the promoters must have read this buffer's previous partial
              if (!mbar_wait(&sh->pempty[buf], ((group >> 1) & 1) ^ 1, 2, sp.wait_limit_ns)) {
                stop = true;
                break;
              }
              tc_fence_after();
            }
            const int st = it % STAGES;
            if (!mbar_wait(&sh->split[st], (it / STAGES) & 1, 3, sp.wait_limit_ns)) {
              stop = true;
              break;
            }
            tc_fence_after();
            const uint32_t a_hi = smem_u32(smem + st * STAGE_BYTES), a_lo = a_hi + A_BYTES;
            const uint32_t b_hi = a_hi + 2 * A_BYTES, b_lo = b_hi + B_BYTES;
  #pragma unroll
            for (int kk = 0; kk < BK / 8; kk++) {
              const uint64_t dah = operand_desc<A_MN>(a_hi, kk), dal = operand_desc<A_MN>(a_lo, kk);
              const uint64_t dbh = operand_desc<B_MN>(b_hi, kk), dbl = operand_desc<B_MN>(b_lo, kk);
              const uint32_t d = tmem + buf * BUF_COLS;
              mma_tf32_pair(d, dal, dbh, idesc, (group_start && kk == 0) ? 0u : 1u);
              mma_tf32_pair(d, dah, dbl, idesc, 1u);
              mma_tf32_pair(d, dah, dbh, idesc, 1u);
            }
            mma_commit_pair(&sh->empty[st]);  // frees the slot in both CTAs
            if ((kt - kb) % GROUP == GROUP - 1 || kt == ke - 1) {
              mma_commit_pair(&sh->pfull[buf]);
              group++;
            }
          }
        }
        if (stop) *failed = 1;
        // Every MMA must be complete before the pair frees its tensor memory.
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&sh->mma_done))
                     : "memory");
        mbar_wait(&sh->mma_done, 0, 6, kTimeoutNs);
      }
    } else if (warp >= SPLIT_WARP0 && warp < SPLIT_WARP0 + STAGES) {
      // ---- splitters (both CTAs): this warp owns ring slot st, i.e. every
      // STAGES-th slice, starting with slice st.
      const int st = warp - SPLIT_WARP0;
      int total = 0;  // slices this pair streams
      for (int u = pair; u < units; u += pairs) {
        int t, kb, ke;
        unit_of(u, tiles, sp, num_k, t, kb, ke);
        total += ke - kb;
      }
      for (int it = st; it < total; it += STAGES) {
        if (__shfl_sync(0xffffffffu, *failed, 0)) break;
        if (!mbar_wait(&sh->full[st], (it / STAGES) & 1, 4, sp.wait_limit_ns)) {
          *failed = 1;
          break;
        }
        uint8_t* stage = smem + st * STAGE_BYTES;
        split_tf32((float4*)stage, (float4*)(stage + A_BYTES), A_BYTES / 16, lane);
        split_tf32((float4*)(stage + 2 * A_BYTES), (float4*)(stage + 2 * A_BYTES + B_BYTES), B_BYTES / 16, lane);
        fence_async_shared();  // generic-proxy writes -> visible to the tensor core
        if (!(sp.withhold_arrive && it == 0 && st == 0 && leader)) mbar_arrive_rank(&sh->split[st], 0);
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_HIGH));
    // ---- promoters and epilogue (both CTAs): TMEM lanes 32*(warp%4)..+31 are
    // this warp's rows, columns [128*h, 128*h + 128) its half of the tile.
    // Every decision below is warp-uniform: tcgen05.ld is .sync.aligned.
    const int q = warp & 3, h = (warp - 8) >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + 128 * h;
    float* xpose = (float*)(smem + EPI_OFFSET) + (warp - 8) * 32 * EPI_LD;
    int group = 0;
    for (int u = pair; u < units && !__shfl_sync(0xffffffffu, *failed, 0); u += pairs) {
      int t, kb, ke;
      const int sidx = unit_of(u, tiles, sp, num_k, t, kb, ke);
      // a split unit's partial tile in the workspace (row-major 256 x 256)
      float* part = sidx < 0 ? nullptr
                             : sp.ws + ((int64_t)sidx * (tiles - sp.whole) + (t - sp.whole)) * TILE_ELEMS +
                                   (int64_t)(rank * BM + 32 * q) * BN + 128 * h + lane;
      const int groups = (ke - kb + GROUP - 1) / GROUP;
      const int mt = t / n_tiles, nt = t % n_tiles;
      // The running total starts at +0 and every partial is added with
      // round-to-nearest, like the reference's c = 0; c += a*b.
      float tot[128];
#pragma unroll
      for (int i = 0; i < 128; i++) tot[i] = 0.0f;
      bool ok = true;
      for (int g = 0; g < groups; g++, group++) {
        const uint32_t buf = (uint32_t)(group & 1);
        if (!__all_sync(0xffffffffu, mbar_wait(&sh->pfull[buf], (group >> 1) & 1, 7, sp.wait_limit_ns))) {
          *failed = 1;
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < 4; j++) {
          float p[32];
          tmem_load32(lane_base + buf * BUF_COLS + 32 * j, p);
#pragma unroll
          for (int i = 0; i < 32; i++) tot[32 * j + i] = __fadd_rn(tot[32 * j + i], p[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_rank(&sh->pempty[buf], 0);  // the buffer may be overwritten
      }
      if (!ok) break;
      // Epilogue: four 32 x 32 blocks through the transpose buffer (the
      // switch keeps the register indices static in a loop that is not
      // unrolled, so the block's code exists once).
      const int64_t m0 = (int64_t)mt * 2 * BM + rank * BM + 32 * q;
#pragma unroll 1
      for (int j = 0; j < 4; j++) {
        switch (j) {
#define GT_XPOSE_CASE(J)                                                          \
  case J:                                                                         \
    _Pragma("unroll") for (int i = 0; i < 32; i++) xpose[lane * EPI_LD + i] = tot[32 * J + i]; \
    break;
          GT_XPOSE_CASE(0)
          GT_XPOSE_CASE(1)
          GT_XPOSE_CASE(2)
          GT_XPOSE_CASE(3)
#undef GT_XPOSE_CASE
        }
        __syncwarp();
        if (!part) {
          epilogue_block<EK>(epi, s, xpose, lane, m0, (int64_t)nt * BN + 128 * h + 32 * j + lane);
        } else {
#pragma unroll 4
          for (int r = 0; r < 32; r++) part[r * BN + 32 * j] = xpose[r * EPI_LD + lane];
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
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 2-D fp32 tensor map over `outer` rows of `inner` contiguous elements with a
// pitch of `ld` elements; zero fill outside. K-major operands: box 16 x 128
// with the 64-byte swizzle; M/N-major: box 32 x 16 with the 128-byte swizzle
// of 32-byte atoms.
static char* make_map(gt_ctx* ctx, CUtensorMap* map, const float* base, int64_t inner, int64_t outer, int64_t ld,
                      bool mn_major) {
  auto encode = (EncodeTiledFn)ctx->encode_tiled;
  if (!encode) return errorf("gemm_tc: cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {mn_major ? 32u : (cuuint32_t)BK, mn_major ? (cuuint32_t)BK : (cuuint32_t)BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                      mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_64B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return errorf("gemm_tc: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return nullptr;
}

// SM pairs a GEMM may occupy: all of them, less the SMs reserved for kernels
// that run beside it (a collective on another stream).
static int64_t pairs_available(const gt_ctx* ctx) {
  const int64_t free_sms = (int64_t)ctx->sm_count - ctx->gemm_sm_reserve;
  return free_sms >= 2 ? free_sms / 2 : 1;
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
  auto kern = gemm_tf32x3_pair_kernel<A_MN, B_MN, EK>;
  static bool configured[64] = {};
  if (ctx->device < 0 || ctx->device >= 64 || !configured[ctx->device]) {
    GT_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    if (ctx->device >= 0 && ctx->device < 64) configured[ctx->device] = true;
  }
  const int64_t tiles = ceil_div(s.M, 2 * BM) * ceil_div(s.N, BN);
  const int64_t units = sp.whole + (tiles - sp.whole) * sp.splits;
  const int64_t avail = pairs_available(ctx);
  const int64_t pairs = units < avail ? units : avail;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = ctx->stream;
  GT_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, s, epi, sp));
  GT_LAUNCH_CHECK();
  return nullptr;
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
    case EK_MASKBITS: return launch_layout<EK_MASKBITS>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    case EK_PLAIN: return launch_layout<EK_PLAIN>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    case EK_BIAS_RELU: return launch_layout<EK_BIAS_RELU>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    case EK_MASK: return launch_layout<EK_MASK>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    case EK_CONV: return launch_layout<EK_CONV>(ctx, s, A, B, epi, a_mn, b_mn, sp);
    default: return launch_layout<EK_GENERIC>(ctx, s, A, B, epi, a_mn, b_mn, sp);
  }
}

// C of the split tiles = epilogue(sum of their partials), the partials added
// in split order, so the result does not depend on which unit finished first.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, SplitPlan sp, int tiles, int n_tiles, int64_t M,
                                     int64_t N, Epi<float> epi) {
  const int rest = tiles - sp.whole;
  const int64_t total = (int64_t)rest * TILE_ELEMS;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / TILE_ELEMS);
    const int64_t e = i - (int64_t)r * TILE_ELEMS;
    const int t = sp.whole + r;
    const int64_t m = (int64_t)(t / n_tiles) * 2 * BM + e / BN, n = (int64_t)(t % n_tiles) * BN + e % BN;
    if (m >= M || n >= N) continue;
    float acc = ws[i];
    for (int k = 1; k < sp.splits; k++) acc = __fadd_rn(acc, ws[(int64_t)k * total + i]);
    epi.store(m, n, acc);
  }
}

// The same with a ReLU bit mask: a thread finishes one column of 32 rows of
// a split tile (consecutive threads, consecutive columns) and writes its word.
__global__ void splitk_reduce_bits_kernel(const float* __restrict__ ws, SplitPlan sp, int tiles, int n_tiles,
                                          int64_t M, int64_t N, Epi<float> epi) {
  const int rest = tiles - sp.whole;
  const int64_t total = (int64_t)rest * TILE_ELEMS;
  const int64_t units = total / 32;  // (tile, 32-row block, column)
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(u / (TILE_ELEMS / 32));
    const int64_t v = u - (int64_t)r * (TILE_ELEMS / 32);
    const int rb = (int)(v / BN), c = (int)(v % BN);
    const int t = sp.whole + r;
    const int64_t m0 = (int64_t)(t / n_tiles) * 2 * BM + 32 * rb, n = (int64_t)(t % n_tiles) * BN + c;
    if (m0 >= M || n >= N) continue;
    uint32_t w = 0;
    for (int j = 0; j < 32 && m0 + j < M; j++) {
      const int64_t i = (int64_t)r * TILE_ELEMS + (int64_t)(32 * rb + j) * BN + c;
      float acc = ws[i];
      for (int k = 1; k < sp.splits; k++) acc = __fadd_rn(acc, ws[(int64_t)k * total + i]);
      const float y = epi.finish(m0 + j, n, acc);
      epi.put(m0 + j, n, y);
      w |= (uint32_t)(y > 0.0f) << j;
    }
    epi.bits_out[(m0 >> 5) * epi.ldw + n] = w;
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

static SplitPlan choose_plan(int64_t tiles, int64_t pairs, int64_t num_k) {
  SplitPlan best;
  best.whole = (int)tiles;
  if (g_force_splits > 1) {
    best.whole = 0;
    best.splits = (int)std::min<int64_t>(g_force_splits, std::max<int64_t>(num_k, 1));
    return best;
  }
  constexpr double kUnitOverhead = 40.0;
  auto reduce_cost = [&](int64_t split_tiles, int S) {
    return (S + 1) * (double)split_tiles * TILE_ELEMS * 4.0 / 5e6 / 0.54;
  };
  const double base = std::ceil((double)tiles / pairs) * (num_k + kUnitOverhead);
  double best_cost = base;
  for (int S = 2; S <= 64 && num_k / S >= 2 * GROUP; S++) {
    // every tile split (the workspace holds S partial tiles per tile: at most 1 GB)
    double c = (double)S * tiles * TILE_ELEMS * 4 > (double)(1ull << 30)
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

char* gemm_tc_f32(gt_ctx* ctx, const GemmShape& s, const float* A, const float* B, const Epi<float>& epi,
                  bool* done) {
  *done = false;
  // TMA needs 16-byte aligned bases and row pitches; tiny problems stay on SIMT.
  if (((uintptr_t)A & 15) || ((uintptr_t)B & 15) || (s.lda & 3) || (s.ldb & 3)) return nullptr;
  if (s.M < 1 || s.N < 1 || s.K < 1 || s.M > INT32_MAX / 2 || s.N > INT32_MAX / 2 || s.K > INT32_MAX / 2)
    return nullptr;
  if (ctx->sm_count < 2) return nullptr;
  if (gemm_path() != 2 && s.M * s.N * s.K < (int64_t)1 << 21) return nullptr;
  const bool a_mn = s.trans_a, b_mn = !s.trans_b;
  const int64_t tiles = ceil_div(s.M, 2 * tc::BM) * ceil_div(s.N, tc::BN);
  const int64_t n_tiles = ceil_div(s.N, tc::BN);
  tc::SplitPlan sp = tc::choose_plan(tiles, tc::pairs_available(ctx), ceil_div(s.K, tc::BK));
  sp.wait_limit_ns = tc::g_wait_limit_ns;
  sp.withhold_arrive = tc::g_withhold_next;
  tc::g_withhold_next = 0;
  char* err;
  if (sp.splits > 1) {
    const int64_t rest = tiles - sp.whole;
    void* ws = nullptr;
    GT_TRY(scratch(ctx, (size_t)sp.splits * rest * tc::TILE_ELEMS * sizeof(float), &ws));
    sp.ws = (float*)ws;
    // Whole tiles finish with their own epilogue; the split tiles' partials
    // go to the workspace and are summed, in order, by the second kernel.
    err = tc::launch_kind(ctx, s, A, B, epi, a_mn, b_mn, sp);
    if (!err) {
      if (epi.bits_out)
        tc::splitk_reduce_bits_kernel<<<grid_for(ctx, rest * tc::TILE_ELEMS / 32, 256), 256, 0, ctx->stream>>>(
            sp.ws, sp, (int)tiles, (int)n_tiles, s.M, s.N, epi);
      else
        tc::splitk_reduce_kernel<<<grid_for(ctx, rest * tc::TILE_ELEMS, 256), 256, 0, ctx->stream>>>(
            sp.ws, sp, (int)tiles, (int)n_tiles, s.M, s.N, epi);
      count_launch();
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) err = cuda_error(e, "splitk_reduce_kernel launch", __FILE__, __LINE__);
    }
    release(ctx, ws);
    if (!err) *done = true;
    return err;
  }
  err = tc::launch_kind(ctx, s, A, B, epi, a_mn, b_mn, sp);
  if (!err) *done = true;
  return err;
}

}  // namespace gt
