// gemm_tc.cu - the persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
// C = alpha * op(A) op(B) + beta * C, column-major, f16/bf16 inputs (kind::f16) or f32 inputs on the
// TF32 path (kind::tf32), fp32 accumulation in tensor memory, f32/f16/bf16 C. Replaces the
// reference's wmma + cp.async template tinyblas_gemm_tc2 and its 24 entry points
// (cuda-shim/libtinycublas/gemm.cu:241-415) and the first-cut tinyblas_gemm_f16_tc / f32_tc
// (gemm.cu:61-221) for every aligned operand.
//
// Shape of one CTA (352 threads, one per SM, persistent over output tiles):
//   warp 0      TMA producer of A, warp 2 TMA producer of B: one thread each streams its operand's k-blocks
//               (128-byte rows, 128B swizzle) into a STAGES-deep shared-memory ring; the bytes complete
//               full[s] by transaction count.
//   warp 1      owns tensor memory (2 x BN columns: two accumulators); one thread issues tcgen05.mma for
//               each k-block, then tcgen05.commit frees the smem stage (empty[s]); after a tile's last
//               k-block a commit publishes the accumulator (tfull[a]).
//   warps 3..10 epilogue, two groups of four (one warp per TMEM lane quadrant): tcgen05.ld 32 lanes x 32
//               columns at a time from the accumulator, apply alpha/beta, convert, store to column-major C
//               (staged TMA stores, or per lane: consecutive lanes hold consecutive rows), then release the
//               accumulator (tempty[a]). Group g drains accumulator g, i.e. every other tile.
// The two accumulators let the epilogue of tile i overlap the main loop of tile i+1, and the two epilogue groups
// let the drains of consecutive tiles overlap each other (output-bound GEMMs).
//
// Tiles: 128 x BN on one CTA (BN 32..256), or 256 x BN (BN 128 or 256) on a cluster of two CTAs with
// tcgen05.mma.cta_group::2 (each CTA loads its 128 rows of A and half of B's BN columns; the even CTA's
// MMA thread drives both tensor cores; each CTA drains its own rows). For GEMMs whose tiles leave SMs
// idle, the k split doubles the CTAs on a tile: one tile per cluster of two CTAs (or two CTA pairs), each
// half running half of the k-blocks, the partial sums exchanged through distributed shared memory. Work units, walked identically by
// every role: output tiles of a plain GEMM, of a strided batch (rank-3 tensor maps, batch = third
// coordinate; stride 0 broadcasts) or of a pointer-array batch (per-element maps written on the device by
// tb200_ptr_maps_kernel), or the per-expert tiles of a grouped GEMM (tile_coord). The epilogue can also
// store each tile into several replicas of C (peers' memory over NVLink) or to an NVLink multicast
// address: the N-sharded GEMM's exchange.
//
// Operand layouts (no transposes materialised): op(A) is K-major when A is stored k x m (op T, the
// ggml call) and MN-major when stored m x k (op N); op(B) is K-major when B is stored k x n (op N)
// and MN-major when stored n x k (op T). Both majors are fed to the tensor core through the
// instruction descriptor's major bits and matching smem descriptors.
//
// Every wait is bounded (an abort flag, an error word, drained copies, freed tensor memory), and the
// kernel is launched with programmatic stream serialization: its set-up overlaps the previous kernel's
// tail and its first memory access waits in griddepcontrol.wait.
//
// No TMA multicast anywhere: every CTA loads its own tiles, and L2 absorbs the reuse.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include "tb200_internal.h"
#include "tb200_device.cuh"

using namespace tb200;

__device__ int g_tb200_err;  // error word: 1 = a pipeline wait gave up

namespace {

constexpr int TC_BM = 128;
// 11 warps: the A producer (warp 0), the MMA issuer (1), the B producer (2), and two epilogue groups of four
// warps (3-6 and 7-10), each warp on TMEM lane quadrant warp % 4. 352 threads leave 186 registers a thread.
constexpr int TC_THREADS = 352;
constexpr int TC_EPI_WARP0 = 3;  // first epilogue warp
constexpr int TC_EPI_WARPS = 8;
// wait budgets in SM cycles (about 2 s and 0.2 s at 2 GHz): far beyond any legitimate wait
constexpr uint64_t WAIT_BUDGET_CYC = 4000000000ull;
constexpr uint64_t DRAIN_BUDGET_CYC = 400000000ull;

struct TcParams {
  int m, n, k, batch;
  int num_kb;                // k-blocks of bk = KC * epr elements
  int m_tiles, n_tiles;
  long long tiles_per_batch, total_tiles;
  int group_m;
  float alpha, beta;
  void *C;
  int ldc;
  long long sC;
  int out_type;
  int a_mn, b_mn;            // 1 = MN-major smem tile (m or n contiguous)
  int a_batched, b_batched;  // rank-3 tensor map
  uint32_t idesc;
  // smem descriptor strides (bytes) of each operand, and the byte offset of UMMA step kk inside a
  // stage: (kk / 4) * cstride + (kk % 4) * kstep
  uint32_t a_lbo, a_sbo, b_lbo, b_sbo;
  uint32_t a_cstride, a_kstep, b_cstride, b_kstep;
  int epr;   // elements per 128-byte row: 64 for 16-bit, 32 for f32
  int bk;    // k elements per stage
  int nrep, row0;  // replicated output: rows go to row0 + row of each of nrep replicas (beta == 0)
  void *rep[8];
  float *mc;       // or of the multicast address of all ranks' f32 C (one store reaches every replica)
  // pointer-array batches: per batch element b, maps[2b] (A) and maps[2b+1] (B) in global memory, C from
  // Carr[b]; the launch does nothing if *skip == skip_gen (the prep kernel found a pointer unfit for TMA in this
  // call, whose generation number that is: the general kernel runs)
  const CUtensorMap *maps;
  void *const *Carr;
  const int *skip;
  int skip_gen;
  // grouped GEMM (MoE experts): when groups > 0, group g owns columns [grp_off[g], grp_off[g + 1]) of B and
  // of C (device offsets, read by the kernel and clamped to [0, n]) and is batch element g of A; its tiles
  // are numbered after those of groups 0 .. g-1, m-tile fastest
  const int *grp_off;
  int groups;
  // grouped GEMM with the token gather fused (K-major B, single-CTA tiles of BN <= 64): column j of B is
  // column gidx[j] of the n_src-column activations the B map covers, loaded with tile::gather4; an id
  // outside [0, n_src) is read as column 0 and its column of the product is zero
  const int *gidx;
  int n_src;
  // epilogue through TMA stores (a third tensor map, of C): each epilogue warp stages its 32 rows x 32 columns in
  // shared memory and one lane stores them as one tiled copy into this GPU's own C (plain GEMMs and strided
  // batches with beta == 0; the map covers m x n (x batch), so rows and columns past the ends are clipped)
  int c_tma, c_batched;
  int epi_pipe;  // plain f32 per-lane stores in 16-column halves, the next half's TMEM load in flight
  // bounded waits: budget of every pipeline wait in SM cycles (WAIT_BUDGET_CYC unless a test shortens it), and
  // the test-only stall: the MMA thread first waits on a barrier nothing arrives at, so that its wait runs out
  uint64_t wait_budget;
  int test_stall;
};

constexpr int TC_MAX_GROUPS = TB200_MAX_GROUPS;

// KC = 128-byte k-chunks per stage. One stage holds A (128 rows) and B (BN rows) for KC * epr values of
// k. The producers and the MMA thread spend a few hundred cycles of issue latency per stage whatever its
// size, so narrow tiles take two chunks per stage to keep the tensor core fed.
template <int BN, int KC, int CG>
struct TcCfg {
  static constexpr int B_ROWS = BN / CG;  // a pair splits B's BN columns between its two CTAs
  static constexpr int A_BYTES = TC_BM * 128 * KC;
  static constexpr int B_BYTES = B_ROWS * 128 * KC;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES_RAW = 196608 / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  // epilogue staging, 32 x 32 f32 per epilogue warp; a grouped GEMM (which never stages: no TMA stores) keeps its
  // column offsets and tile-count prefix there instead
  static constexpr int STG_BYTES = TC_EPI_WARPS * 4096;
  static constexpr int GRP_BYTES = 2 * 4 * (TC_MAX_GROUPS + 1);
  static_assert(GRP_BYTES <= STG_BYTES, "the grouped GEMM's tables live in the staging area");
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES;
};


__device__ __forceinline__ void decode_tile(const TcParams &p, long long t, int &b, int &mt, int &nt) {
  b = (int)(t / p.tiles_per_batch);
  long long r = t - (long long)b * p.tiles_per_batch;
  const long long group_tiles = (long long)p.group_m * p.n_tiles;
  const int g = (int)(r / group_tiles);
  const int first_m = g * p.group_m;
  int gm = p.m_tiles - first_m;
  if (gm > p.group_m) gm = p.group_m;
  const int local = (int)(r - (long long)g * group_tiles);
  mt = first_m + local % gm;
  nt = local / gm;
}

// One output tile: batch element (or group) b, m-tile mt, and its columns [n0, n_end) of B and C (absolute,
// so that a grouped GEMM's tile can start inside B).
struct TileCoord {
  int b, mt, n0, n_end;
};

// tile t of a plain or strided/pointer-array GEMM (grouped raster inside each batch element), or of a grouped
// GEMM (g_off / g_pre: the groups' clamped column offsets and tile-count prefix in shared memory)
template <int BN>
__device__ __forceinline__ TileCoord tile_coord(const TcParams &p, long long t, const int *g_off, const int *g_pre) {
  TileCoord c;
  if (p.groups > 0) {
    int lo = 0, hi = p.groups - 1;  // the group whose tile range holds t: g_pre[g] <= t < g_pre[g + 1]
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (g_pre[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    const int local = (int)(t - g_pre[lo]);
    c.b = lo;
    c.mt = local % p.m_tiles;
    c.n0 = g_off[lo] + (local / p.m_tiles) * BN;
    c.n_end = g_off[lo + 1];
    return c;
  }
  int nt;
  decode_tile(p, t, c.b, c.mt, nt);
  c.n0 = nt * BN;
  c.n_end = p.n;
  return c;
}

// One operand's loads for one stage: `rows` (128 for A, BN/CG for B) x KC chunks. K-major: chunk c is a
// rows x 128-byte box at k0 + c*epr. MN-major: rows/epr boxes of epr (m or n) x KC*epr k-rows. With
// CG == 2 the bytes complete on the pair's even CTA's barrier (shared::cluster address bar2).
template <int KC, int CG>
__device__ __forceinline__ void load_operand(uint8_t *dst, const CUtensorMap *tm, uint64_t *bar, uint32_t bar2,
                                             int mn_major, int batched, int rows, int epr, int mn0, int k0, int b) {
  auto ld = [&](uint8_t *d, int c0, int c1) {
    if (CG == 1) {
      if (batched) tma_load_3d(d, tm, bar, c0, c1, b);
      else tma_load_2d(d, tm, bar, c0, c1);
    } else {
      if (batched) tma_load_3d_cg2(d, tm, bar2, c0, c1, b);
      else tma_load_2d_cg2(d, tm, bar2, c0, c1);
    }
  };
  if (!mn_major) {
#pragma unroll
    for (int c = 0; c < KC; ++c) ld(dst + c * rows * 128, k0 + c * epr, mn0);
  } else {
    for (int j = 0; j < rows / epr; ++j) ld(dst + j * KC * epr * 128, mn0 + j * epr, k0);
  }
}

// CG = 1: one CTA per 128 x BN tile. CG = 2: two CTAs per 256 x BN tile (2-SM UMMA, the pair of cluster ranks
// that differ in bit 0): each CTA loads its 128 rows of A and BN/2 rows of B, the even CTA's MMA thread
// drives both tensor cores, and each CTA's epilogue drains its own 128 rows from its own tensor memory.
// KS = 2: the k split. Each tile gets a second CTA (CG = 1) or a second pair (CG = 2), one tile per cluster,
// and each half of the cluster runs half of the k-blocks into its own accumulator. Each CTA then finalises
// half of its rows' columns: it parks its partial sums of the other half in its idle operand ring (one tile:
// every load consumed, every MMA committed), and reads the peer's parked sums of its own half over
// distributed shared memory, adds them and stores C. No workspace and no L2 round trip, and each CTA
// drains half of the tile.
template <int KIND, int BN, int KC, int CG, int KS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tb200_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  using Cfg = TcCfg<BN, KC, CG>;
  constexpr int STAGES = Cfg::STAGES;
  static_assert(KS == 1 || (BN >= 64 && STAGES * Cfg::STAGE_BYTES >= TC_BM * (BN / 2) * 4),
                "k split: the operand ring must hold 128 x BN/2 f32 partial sums");
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment of the shared-window offset: the 128B swizzle atom is 8 rows x 128 bytes. The
  // offset is the same in both CTAs of a pair, as the 2-SM UMMA requires.
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *smA = smem;
  uint8_t *smB = smem + STAGES * Cfg::A_BYTES;
  uint8_t *stg_all = smem + STAGES * Cfg::STAGE_BYTES;  // epilogue staging, 4 KB per epilogue warp
  uint64_t *bars = (uint64_t *)(stg_all + Cfg::STG_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *tfull = bars + 2 * STAGES;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint64_t *xfull = drain + 1;  // KS = 2: the k-split peer has parked its partial sums of this CTA's columns
  uint32_t *tmem_slot = (uint32_t *)(drain + 2);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);
  int *g_off = (int *)stg_all;             // grouped GEMM: clamped column offsets ...
  int *g_pre = g_off + TC_MAX_GROUPS + 1;  // ... and tile-count prefix

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int CSIZE = CG * KS;   // CTAs per tile, launched as one cluster
  constexpr bool CL = CSIZE > 1;
  const uint32_t crank = CL ? cluster_ctarank() : 0u;
  const uint32_t rank = CG == 2 ? (crank & 1u) : 0u;                  // the CTA's half of a pair tile's rows
  const uint32_t kslice = KS == 2 ? (CG == 2 ? crank >> 1 : crank) : 0u;  // the CTA's half of the k-blocks
  const uint32_t pair_even = crank & ~1u, pair_odd = crank | 1u;      // cluster ranks of the CTA's pair
  const uint32_t xpeer = crank ^ (CG == 2 ? 2u : 1u);                 // the CTA with the same rows, other k half
  const bool leader = rank == 0;
  // tile index stream: one per CTA, or one per cluster
  const long long t_first = (long long)(blockIdx.x / CSIZE);
  const long long t_step = (long long)(gridDim.x / CSIZE);
  const int kb_lo = KS == 2 ? (int)((long long)kslice * p.num_kb / 2) : 0;
  const int kb_hi = KS == 2 ? (int)((long long)(kslice + 1) * p.num_kb / 2) : p.num_kb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 2);  // one arrive.expect_tx from each producer (of the even CTA, for a pair)
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4 * CG);  // every epilogue warp of the tile
    }
    mbar_init(drain, 1);
    mbar_init(xfull, 32 * TC_EPI_WARPS);  // every epilogue thread of the k-split peer
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (p.c_tma) prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    if (CG == 1) {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    } else {
      tmem_alloc_cg2(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_cg2();
    }
  }
  tc_fence_before();
  __syncwarp();                 // barrier.cluster.*.aligned wants every warp converged
  if (CL) cluster_sync();  // peers' loads, commits and arrivals target this CTA's barriers: all initialised
  else __syncthreads();
  tc_fence_after();
  // Everything above touched only this CTA's own resources and the kernel parameters, and may overlap the
  // end of the kernel before this one in the stream. From here on operands and C are read and written:
  // wait for that kernel to complete. Then let the next kernel set up on the SMs this one leaves free.
  griddep_wait();
  griddep_launch_dependents();
  long long total_tiles = p.total_tiles;
  // pointer-array batch with some pointer unfit for TMA (the flag written by the prep kernel before this one, read
  // once that kernel has completed): no tiles, every role falls through to the teardown, the general kernel
  // launched behind this one computes the batch
  if (p.skip && *(volatile const int *)p.skip == p.skip_gen) total_tiles = 0;
  if (p.groups > 0) {
    // the groups' columns, clamped so that no tile reaches outside B or C whatever the offsets hold, and the
    // prefix of their tile counts (the same in every CTA)
    for (int g = threadIdx.x; g <= p.groups; g += blockDim.x) {
      int o = p.grp_off[g];
      g_off[g] = o < 0 ? 0 : o > p.n ? p.n : o;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int acc = 0, lo = 0;
      for (int g = 0; g < p.groups; ++g) {
        g_pre[g] = acc;
        lo = g_off[g] > lo ? g_off[g] : lo;  // columns before the previous group's start count as empty
        const int hi = g_off[g + 1] > lo ? g_off[g + 1] : lo;
        g_off[g] = lo;
        acc += ((hi - lo + BN - 1) / BN) * p.m_tiles;
      }
      g_pre[p.groups] = acc;
      if (g_off[p.groups] < lo) g_off[p.groups] = lo;
    }
    __syncthreads();
    total_tiles = g_pre[p.groups];
  }
  const uint32_t tmem_base = *tmem_slot;
  // shared::cluster addresses of the even CTA's barriers (CG == 2)
  const uint32_t lead_full0 = CG == 2 ? mapa_shared(smem_u32(full), pair_even) : 0u;
  const uint32_t lead_tempty0 = CG == 2 ? mapa_shared(smem_u32(tempty), pair_even) : 0u;

  constexpr int NG = KC * BN / 4;  // tile::gather4 loads of B per stage (fused token gather)
  if (warp == 2 && CG == 1 && NG <= 32 && p.gidx != nullptr) {
    // ------------------------------------------------------------------ B producer, fused token gather
    // Lane l < NG issues one gather4 a stage: k-chunk l / (BN / 4), B rows 4 (l % (BN / 4)) .. + 3 of the
    // tile, i.e. the tile's columns of B, each read from the source column its token id names (an id
    // outside [0, n_src) reads column 0, and the epilogue zeroes that column; columns past n are not stored).
    const int gc = lane / (BN / 4), gi = lane % (BN / 4);
    int s = 0;
    uint32_t ph = 0;
    uint32_t issued = 0, issued_par = 0;
    for (long long t = t_first; t < total_tiles; t += t_step) {
      // lane 0 reads the abort flag for the warp: every lane leaves the loop on the same tile (the loop
      // body's shuffles need all 32)
      const int go = __shfl_sync(0xffffffffu, lane == 0 ? (*abort_flag ? 0 : 1) : 0, 0);
      if (!go) break;
      const TileCoord tc = tile_coord<BN>(p, t, g_off, g_pre);
      int rid[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int col = tc.n0 + 4 * gi + q;
        const int id = lane < NG && col < p.n ? __ldg(p.gidx + col) : 0;
        rid[q] = id >= 0 && id < p.n_src ? id : 0;
      }
      bool ok = true;
      for (int kb = kb_lo; kb < kb_hi; ++kb) {
        int got = 1;
        if (lane == 0) {
          got = mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.wait_budget) ? 1 : 0;
          if (got) mbar_arrive_expect_tx(&full[s], (uint32_t)Cfg::B_BYTES);
        }
        got = __shfl_sync(0xffffffffu, got, 0);  // also orders the expect_tx before every lane's copy
        if (!got) {
          ok = false;
          break;
        }
        if (lane < NG)
          tma_gather4(smB + s * Cfg::B_BYTES + gc * Cfg::B_ROWS * 128 + gi * 512, &tmB, &full[s],
                      kb * p.bk + gc * p.epr, rid[0], rid[1], rid[2], rid[3]);
        issued |= 1u << s;
        issued_par = (issued_par & ~(1u << s)) | (ph << s);
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
    }
    if (lane == 0 && *abort_flag) {  // let every copy still in flight land before shared memory goes away
      volatile int no_abort = 0;
      for (int q = 0; q < STAGES; ++q)
        if (issued & (1u << q)) (void)mbar_wait(&full[q], (issued_par >> q) & 1u, &no_abort, DRAIN_BUDGET_CYC);
    }
  } else if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------------ TMA producers (A: warp 0, B: warp 2)
    if (lane == 0) {
      const bool is_a = warp == 0;
      const CUtensorMap *tm0 = is_a ? &tmA : &tmB;
      uint8_t *base = is_a ? smA : smB;
      const int stage_bytes = is_a ? Cfg::A_BYTES : Cfg::B_BYTES;
      const int rows = is_a ? TC_BM : Cfg::B_ROWS;
      const int mn_major = is_a ? p.a_mn : p.b_mn;
      const int batched = is_a ? p.a_batched : p.b_batched;
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued = 0, issued_par = 0;  // per stage: a fill is outstanding, and its phase parity
      for (long long t = t_first; t < total_tiles && !*abort_flag; t += t_step) {
        const TileCoord tc = tile_coord<BN>(p, t, g_off, g_pre);
        const int b = tc.b;
        const int mn0 = is_a ? tc.mt * (TC_BM * CG) + (int)rank * TC_BM : tc.n0 + (int)rank * Cfg::B_ROWS;
        const CUtensorMap *tm = tm0;
        if (p.maps) {  // this batch element's own map, written by the prep kernel through the generic proxy
          tm = p.maps + 2 * b + (is_a ? 0 : 1);
          fence_tensormap_acquire(tm);
        }
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.wait_budget)) break;
          // the even CTA announces the bytes of both CTAs; the odd CTA's copies only complete them
          if (leader) mbar_arrive_expect_tx(&full[s], (uint32_t)(stage_bytes * CG));
          load_operand<KC, CG>(base + s * stage_bytes, tm, &full[s], lead_full0 + (uint32_t)(s * 8), mn_major,
                               batched, rows, p.epr, mn0, kb * p.bk, b);
          issued |= 1u << s;
          issued_par = (issued_par & ~(1u << s)) | (ph << s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (*abort_flag && leader) {  // let every copy still in flight land before shared memory goes away
        volatile int no_abort = 0;
        for (int q = 0; q < STAGES; ++q)
          if (issued & (1u << q)) (void)mbar_wait(&full[q], (issued_par >> q) & 1u, &no_abort, DRAIN_BUDGET_CYC);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (the even CTA of a pair)
    if (lane == 0 && leader) {
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      // stage-0 descriptors, and per-step offsets in the 16-byte units of the start-address field (the
      // sum stays inside the 14-bit field: shared memory offsets are below 256 KB)
      const uint64_t a_desc0 = smem_desc_sw128(smem_u32(smA), p.a_lbo, p.a_sbo);
      const uint64_t b_desc0 = smem_desc_sw128(smem_u32(smB), p.b_lbo, p.b_sbo);
      uint32_t a_off[4 * KC], b_off[4 * KC];
#pragma unroll
      for (int kk = 0; kk < 4 * KC; ++kk) {
        a_off[kk] = ((kk >> 2) * p.a_cstride + (kk & 3) * p.a_kstep) >> 4;
        b_off[kk] = ((kk >> 2) * p.b_cstride + (kk & 3) * p.b_kstep) >> 4;
      }
      // commit targets: this CTA's barriers, and for a pair the odd CTA's too
      const uint32_t empty0_l = smem_u32(empty), tfull0_l = smem_u32(tfull), drain_l = smem_u32(drain);
      const uint32_t empty0_p = CG == 2 ? mapa_shared(empty0_l, pair_odd) : 0u;
      const uint32_t tfull0_p = CG == 2 ? mapa_shared(tfull0_l, pair_odd) : 0u;
      // test-only (TB200_TEST_STALL=1): a wait that nothing completes - no CTA of a single-CTA, unsplit tile
      // arrives on xfull - runs out of its budget and takes the abort path below
      if (p.test_stall && KS == 1 && CG == 1) (void)mbar_wait(xfull, 0, abort_flag, p.wait_budget);
      for (long long t = t_first; t < total_tiles && !*abort_flag; t += t_step) {
        if (!mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, p.wait_budget)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, p.wait_budget)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad0 = a_desc0 + (uint64_t)((uint32_t)(s * Cfg::A_BYTES) >> 4);
          const uint64_t bd0 = b_desc0 + (uint64_t)((uint32_t)(s * Cfg::B_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4 * KC; ++kk) {  // UMMA_K = 16 (f16/bf16) or 8 (tf32): 4 steps per chunk
            const uint32_t en = kb != kb_lo || kk != 0;  // the first k-block of the slice overwrites
            if (CG == 1) {
              if (KIND == 0) umma_f16(d_tmem, ad0 + a_off[kk], bd0 + b_off[kk], p.idesc, en);
              else umma_tf32(d_tmem, ad0 + a_off[kk], bd0 + b_off[kk], p.idesc, en);
            } else {
              if (KIND == 0) umma_f16_cg2(d_tmem, ad0 + a_off[kk], bd0 + b_off[kk], p.idesc, en);
              else umma_tf32_cg2(d_tmem, ad0 + a_off[kk], bd0 + b_off[kk], p.idesc, en);
            }
          }
          if (CG == 1) {
            umma_commit(&empty[s]);
          } else {
            umma_commit_cg2(empty0_l + (uint32_t)(s * 8));
            umma_commit_cg2(empty0_p + (uint32_t)(s * 8));
          }
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        if (CG == 1) {
          umma_commit(&tfull[acc]);
        } else {
          umma_commit_cg2(tfull0_l + (uint32_t)(acc * 8));
          umma_commit_cg2(tfull0_p + (uint32_t)(acc * 8));
        }
        acc ^= 1;
        if (acc == 0) aph ^= 1u;
      }
      // every MMA issued above has completed once this commit arrives
      if (CG == 1) umma_commit(drain);
      else umma_commit_cg2(drain_l);
      volatile int no_abort = 0;
      (void)mbar_wait(drain, 0, &no_abort, DRAIN_BUDGET_CYC);
    }
  } else if (warp >= TC_EPI_WARP0) {
    // ------------------------------------------------------------------ epilogue (warps 3..10)
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int egrp = (warp - TC_EPI_WARP0) >> 2;  // epilogue group: warps 3-6 and 7-10
    // 32-column chunks this CTA stores: all, or (k split) its half [c_lo, c_lo + HCH); the peer stores
    // [o_lo, o_lo + HCH)
    constexpr int HCH = KS == 2 ? BN / 64 : BN / 32;
    const int c_lo = (int)kslice * HCH;
    const int o_lo = HCH - c_lo;
    // Without the k split the two groups take alternate tiles, group g draining accumulator g, so that one
    // group's stores overlap the other's. With it (one tile per cluster) both groups share the tile, each with
    // half of the chunks (group 0 all of them when there is one).
    const int g_lo = KS == 2 && HCH >= 2 ? egrp * (HCH / 2) : 0;
    const int g_n = KS == 2 ? (HCH >= 2 ? HCH / 2 : (egrp == 0 ? HCH : 0)) : HCH;
    const int acc = KS == 2 ? 0 : egrp;
    uint32_t aph = 0, xph = 0;
    const int osz = p.out_type == 0 ? 4 : 2;
    const long long t_step_g = KS == 2 ? t_step : 2 * t_step;
    for (long long t = t_first + (KS == 2 ? 0 : egrp * t_step); t < total_tiles; t += t_step_g) {
      const TileCoord tc = tile_coord<BN>(p, t, g_off, g_pre);
      const int b = tc.b, mt = tc.mt;
      // one lane waits, the warp follows its verdict: tcgen05.ld below needs the whole warp converged
      int got = 0;
      if (lane == 0) got = mbar_wait(&tfull[acc], aph, abort_flag, p.wait_budget) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      tc_fence_after();
      // TMEM address of 32-column chunk c of this warp's lane quadrant in the current accumulator
      const uint32_t t_chunk0 = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      uint32_t ra[32];
      if (KS == 2) {
        // park the partial sums of the peer's columns (this group's share of them), announce them, wait for the
        // peer's of this CTA's own
        float4 *park = (float4 *)smem;  // [chunk][4 columns][quadrant][lane]: a warp's stores are contiguous
#pragma unroll 1
        for (int c = g_lo; c < g_lo + g_n; ++c) {
          tmem_ld_32x32b_x32(t_chunk0 + (uint32_t)((o_lo + c) * 32), ra);
          tmem_ld_wait_regs(ra);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            park[((c * 8 + q) * 4 + quad) * 32 + lane] =
                make_float4(__uint_as_float(ra[4 * q]), __uint_as_float(ra[4 * q + 1]), __uint_as_float(ra[4 * q + 2]),
                            __uint_as_float(ra[4 * q + 3]));
        }
        mbar_arrive_cluster(mapa_shared(smem_u32(xfull), xpeer));  // every thread releases its own stores
        if (g_n > 0) {
          int parked = 0;
          if (lane == 0) parked = mbar_wait_cluster(xfull, xph, abort_flag, p.wait_budget) ? 1 : 0;
          parked = __shfl_sync(0xffffffffu, parked, 0);
          __syncwarp();  // lane 0's acquire orders the peer's parked sums before every lane's reads
          xph ^= 1u;
          if (!parked) break;
        }
      }
      const int row = mt * (TC_BM * CG) + (int)rank * TC_BM + quad * 32 + lane;
      const int n0 = tc.n0;
      char *Cb = p.Carr ? (char *)p.Carr[b] : (char *)p.C + (p.groups > 0 ? 0ll : (long long)b * p.sC * osz);
      const bool row_ok = row < p.m;
      // one chunk's epilogue: the peer's partial sums added (k split), alpha / beta, conversion, stores
      auto store_chunk = [&](uint32_t(&r)[32], int c) {
        if (KS == 2) {  // own sum + the peer's (two terms: the same value whichever CTA adds them)
          const uint32_t pk = mapa_shared(smem_u32(smem), xpeer);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 v =
                ld_shared_cluster_f4(pk + (uint32_t)(((((c - c_lo) * 8 + q) * 4 + quad) * 32 + lane) * 16));
            r[4 * q] = __float_as_uint(__uint_as_float(r[4 * q]) + v.x);
            r[4 * q + 1] = __float_as_uint(__uint_as_float(r[4 * q + 1]) + v.y);
            r[4 * q + 2] = __float_as_uint(__uint_as_float(r[4 * q + 2]) + v.z);
            r[4 * q + 3] = __float_as_uint(__uint_as_float(r[4 * q + 3]) + v.w);
          }
        }
        const int col0 = n0 + c * 32;
        if (p.c_tma) {
          // stage the warp's 32 rows x 32 columns (column-major, as C) and store them with one TMA copy; rows and
          // columns outside C are clipped by the map. The previous chunk's store must have read the buffer.
          const int wrow = mt * (TC_BM * CG) + (int)rank * TC_BM + quad * 32;
          if (wrow < p.m && col0 < tc.n_end) {
            uint8_t *stg = stg_all + (warp - TC_EPI_WARP0) * 4096;
            if (lane == 0) bulk_wait_read_all();
            __syncwarp();
            if (p.out_type == 0) {
              float *st = (float *)stg;
#pragma unroll
              for (int j = 0; j < 32; ++j) st[j * 32 + lane] = p.alpha * __uint_as_float(r[j]);
            } else if (p.out_type == 1) {
              __half *st = (__half *)stg;
#pragma unroll
              for (int j = 0; j < 32; ++j) st[j * 32 + lane] = __float2half_rn(p.alpha * __uint_as_float(r[j]));
            } else {
              __nv_bfloat16 *st = (__nv_bfloat16 *)stg;
#pragma unroll
              for (int j = 0; j < 32; ++j) st[j * 32 + lane] = __float2bfloat16_rn(p.alpha * __uint_as_float(r[j]));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (p.c_batched) tma_store_3d(&tmC, stg, wrow, col0, b);
              else tma_store_2d(&tmC, stg, wrow, col0);
              bulk_commit();
            }
          }
          return;
        }
        if (p.gidx && col0 < tc.n_end) {  // fused gather: a column whose token id is out of range is zero
          const int cj = col0 + lane;
          const int id = cj < tc.n_end ? __ldg(p.gidx + cj) : 0;
          const unsigned in_range = __ballot_sync(0xffffffffu, id >= 0 && id < p.n_src);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (!((in_range >> j) & 1u)) r[j] = 0u;
        }
        if (row_ok && col0 < tc.n_end) {
          const int ncols = tc.n_end - col0 < 32 ? tc.n_end - col0 : 32;
          if (p.mc) {
            // N-sharded GEMM, multicast: one store per element, replicated to every rank's C by the switch
            float *dst = p.mc + p.row0 + row + (long long)col0 * p.ldc;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < ncols) multimem_st_f32(dst + (long long)j * p.ldc, p.alpha * __uint_as_float(r[j]));
          } else if (p.nrep > 0) {
            // N-sharded GEMM: this rank's rows go straight into every replica of C, peers' over NVLink
            for (int q = 0; q < p.nrep; ++q) {
              char *Cq = (char *)p.rep[q] + (long long)p.row0 * osz;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncols)
                  store_out(Cq, row + (long long)(col0 + j) * p.ldc, p.alpha * __uint_as_float(r[j]), p.out_type);
            }
          } else if (p.beta == 0.f) {
            if (p.out_type == 0 && p.alpha == 1.f) {
              float *dst = (float *)Cb + row + (long long)col0 * p.ldc;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncols) dst[(long long)j * p.ldc] = __uint_as_float(r[j]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < ncols)
                  store_out(Cb, row + (long long)(col0 + j) * p.ldc, p.alpha * __uint_as_float(r[j]), p.out_type);
            }
          } else {
            float old[32];
#pragma unroll
            for (int j = 0; j < 32; ++j)
              old[j] = j < ncols ? load_out(Cb, row + (long long)(col0 + j) * p.ldc, p.out_type) : 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < ncols)
                store_out(Cb, row + (long long)(col0 + j) * p.ldc, p.alpha * __uint_as_float(r[j]) + p.beta * old[j],
                          p.out_type);
          }
        }
      };
      if (KS == 1 && p.epi_pipe && !p.c_tma && p.out_type == 0 && p.beta == 0.f && !p.gidx && !p.nrep && !p.mc) {
        // plain f32 per-lane stores in 16-column halves: the next half's TMEM load is in flight while this half's
        // stores issue (the same 32 registers as one 32-column chunk)
        uint32_t ha[16], hb[16];
        auto store_half = [&](const uint32_t(&h)[16], int hh) {
          const int col0 = n0 + hh * 16;
          if (row_ok && col0 < tc.n_end) {
            const int ncols = tc.n_end - col0 < 16 ? tc.n_end - col0 : 16;
            float *dst = (float *)Cb + row + (long long)col0 * p.ldc;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (j < ncols) dst[(long long)j * p.ldc] = p.alpha * __uint_as_float(h[j]);
          }
        };
        const int h_lo = 2 * (c_lo + g_lo), h_hi = 2 * (c_lo + g_lo + g_n);  // an even count of halves
        tmem_ld_32x32b_x16(t_chunk0 + (uint32_t)(h_lo * 16), ha);
        tmem_ld_wait_regs16(ha);
#pragma unroll 1
        for (int hh = h_lo; hh < h_hi; hh += 2) {
          tmem_ld_32x32b_x16(t_chunk0 + (uint32_t)((hh + 1) * 16), hb);
          store_half(ha, hh);
          tmem_ld_wait_regs16(hb);
          const bool more = hh + 2 < h_hi;
          if (more) tmem_ld_32x32b_x16(t_chunk0 + (uint32_t)((hh + 2) * 16), ha);
          store_half(hb, hh + 1);
          if (more) tmem_ld_wait_regs16(ha);
        }
      } else {
#pragma unroll 1
        for (int c = c_lo + g_lo; c < c_lo + g_lo + g_n; ++c) {
          tmem_ld_32x32b_x32(t_chunk0 + (uint32_t)(c * 32), ra);
          tmem_ld_wait_regs(ra);
          store_chunk(ra, c);
        }
      }
      tc_fence_before();
      __syncwarp();
      // the accumulator is free again once its group's four warps have read it (with the k split, one tile per
      // cluster and nothing more to compute, group 0 alone signals)
      if (lane == 0 && (KS == 1 || egrp == 0)) {
        if (CG == 1) mbar_arrive(&tempty[acc]);
        else mbar_arrive_cluster(lead_tempty0 + (uint32_t)(acc * 8));
      }
      aph ^= 1u;
    }
    if (p.c_tma && lane == 0) bulk_wait_all();  // the staged stores have completed before the CTA leaves
  }

  if ((p.nrep > 0 || p.mc) && warp >= TC_EPI_WARP0) __threadfence_system();  // peers' replicas: stores performed
  tc_fence_before();
  __syncwarp();
  if (CL) cluster_sync();  // no CTA leaves while a peer may still read its memory or signal its barriers
  else __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicExch(&g_tb200_err, 1);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if (CG == 1) tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    else tmem_dealloc_cg2(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace

namespace {

// One thread per batch element of a pointer-array GEMM: copies the template maps (built on the host with a
// placeholder address) to maps[2b] / maps[2b+1], points them at Aarr[b] / Barr[b], and writes the call's
// generation number `gen` to *bad when a pointer is not 16-byte aligned (a TMA source must be) so that the
// tensor-core launch stands down. The flag is never cleared: a later call compares it with its own number.
__global__ void tb200_ptr_maps_kernel(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
                                      const void *const *Aarr, const void *const *Barr, CUtensorMap *maps, int batch,
                                      int *bad, int gen) {
  // launched with programmatic stream serialization: the pointer arrays may come from the kernel before; the
  // tensor-core kernel behind this one may set up meanwhile (it reads the maps only after this grid completes)
  griddep_wait();
  griddep_launch_dependents();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const void *a = Aarr[b];
  const void *bb = Barr[b];
  if ((((uintptr_t)a) | ((uintptr_t)bb)) & 15) atomicExch(bad, gen);
  maps[2 * b] = tA;
  maps[2 * b + 1] = tB;
  tensormap_set_address(&maps[2 * b], a);
  tensormap_set_address(&maps[2 * b + 1], bb);
  fence_tensormap_release();
}

// ---------------------------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static int tried = 0;
  if (!fn && !tried) {
    tried = 1;
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
  }
  return fn;
}

// rank-2 (batch stride 0 or batch 1) or rank-3 tiled map with a 128-byte-wide, 128B-swizzled box
bool make_map(CUtensorMap *tm, CUtensorMapDataType dt, int esz, const void *base, long long d0, long long d1,
              long long ld, int batch, long long bstride, int box0, int box1, int *batched) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return false;
  const bool b3 = batch > 1 && bstride != 0;
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * esz), (cuuint64_t)(bstride * esz)};
  cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(tm, dt, b3 ? 3 : 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  *batched = b3 ? 1 : 0;
  return r == CUDA_SUCCESS;
}

// the C map of the TMA-store epilogue: m x n (x batch) elements of the output type, a 32 x 32 box, no swizzle
bool make_c_map(CUtensorMap *tm, int out_type, void *C, long long m, long long n, long long ldc, int batch,
                long long sC, int *batched) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return false;
  const int esz = out_type == TB200_F32 ? 4 : 2;
  const CUtensorMapDataType dt = out_type == TB200_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : out_type == TB200_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const bool b3 = batch > 1;
  cuuint64_t dims[3] = {(cuuint64_t)m, (cuuint64_t)n, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ldc * esz), (cuuint64_t)(sC * esz)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(tm, dt, b3 ? 3 : 2, C, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  *batched = b3 ? 1 : 0;
  return r == CUDA_SUCCESS;
}

template <int KIND, int BN, int KC, int CG, int KS = 1>
int launch_bn(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tcm, const TcParams &p, int num_sms,
              cudaStream_t s) {
  using Cfg = TcCfg<BN, KC, CG>;
  constexpr int CSIZE = CG * KS;  // CTAs per tile: one cluster
  auto kern = tb200_gemm_tc_kernel<KIND, BN, KC, CG, KS>;
  static int attr_done[64], max_clusters[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    if (CSIZE > 1) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = CSIZE;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(CSIZE * (num_sms / CSIZE), 1, 1);
      cfg.blockDim = dim3(TC_THREADS, 1, 1);
      cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int nc = 0;
      if (cudaOccupancyMaxActiveClusters(&nc, kern, &cfg) != cudaSuccess || nc <= 0) nc = num_sms / CSIZE;
      (void)cudaGetLastError();
      max_clusters[dev] = nc;
    }
    attr_done[dev] = 1;
  }
  const long long slots = CSIZE > 1 ? max_clusters[dev] : num_sms;
  // KS = 2 runs one tile per cluster (partial sums are parked in the operand ring after the only tile)
  if (KS == 2 && p.total_tiles > slots) return (int)cudaErrorNotSupported;
  const long long units = p.total_tiles < slots ? p.total_tiles : slots;
  const unsigned grid = (unsigned)(units * CSIZE);
  if (tb200_trace())
    fprintf(stderr,
            "[trace] launch tb200_gemm_tc<%s,BN=%d,KC=%d,CG=%d%s> grid=(%u,1,1) block=(%d,1,1) smem=%d stages=%d m=%d "
            "n=%d k=%d batch=%d store=%s\n",
            KIND ? "tf32" : "f16", BN, KC, CG, KS == 2 ? ",KS=2" : "", grid, TC_THREADS, Cfg::SMEM_BYTES, Cfg::STAGES,
            p.m, p.n, p.k, p.batch, p.c_tma ? "tma" : "lanes");
  // Programmatic stream serialization: this grid may be scheduled while the kernel before it in the stream
  // finishes (the kernel waits for it with griddep_wait before touching memory), which hides the launch and
  // the set-up of barriers and tensor memory behind that kernel's last tiles.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[2];
  int na = 0;
  if (CSIZE > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = CSIZE;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  if (tb200_pdl()) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(TC_THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = na;
  return (int)cudaLaunchKernelEx(&cfg, kern, ta, tb, tcm, p);
}

// tile width BN -> k-chunks per stage: the widest single-CTA tile keeps one chunk (four stages of 48 KB);
// narrower tiles take two so that each stage carries enough tensor work to cover its issue cost. A pair's
// 256 x 256 tile has 32 KB per CTA per chunk and keeps one chunk (six stages; two, in three stages, for launches
// of three waves or more: launch_tc_impl); its 256 x 128 tile has 24 KB and takes two (four stages of 48 KB).
constexpr int kc_for(int bn) { return bn >= 256 ? 1 : 2; }

}  // namespace

extern "C" int tb200_tc_ok(const tb200_gemm_t *g) {
  const int es = g->in_type == TB200_F32 ? 4 : 2;
  if (g->Aarr || g->Barr || g->Carr) return 0;
  if (g->in_type == TB200_F32 && (g->opA != 1 || g->opB != 0)) return 0;  // TF32: K-major operands only
  if (g->k <= 0) return 0;
  if (((long long)g->lda * es) % 16 || ((long long)g->ldb * es) % 16) return 0;
  if (((uintptr_t)g->A & 15) || ((uintptr_t)g->B & 15)) return 0;
  if (g->batch > 1 && (((g->sA * es) % 16) || ((g->sB * es) % 16))) return 0;
  return 1;
}

// generation number of the last pointer-array launch of this process (read by the allocation-free entry point's
// test hook)
static int g_last_ptr_gen;

// The shared launcher. ptr_ws != NULL: pointer-array batch, scratch laid out as [flag (256 B)][maps]; the flag
// starts at zero when the scratch is made and is never cleared (see tb200_ptr_maps_kernel).
static int launch_tc_impl(const tb200_gemm_t *g, int tile_n, int pair, int num_sms, void *ptr_ws, cudaStream_t s) {
  const bool f32in = g->in_type == TB200_F32;
  const int es = f32in ? 4 : 2;
  const int epr = 128 / es;
  int bn = tile_n;
  if (bn != 32 && bn != 64 && bn != 128 && bn != 256) bn = 128;
  // the fused token gather loads B with tile::gather4 into single-CTA tiles of 32 or 64 columns, K-major
  if (g->gidx) {
    if (f32in || !g->groups || g->opB != 0 || ptr_ws || g->nrep || g->mc || g->n_src < 1)
      return (int)cudaErrorNotSupported;
    pair = 0;
    bn = bn <= 32 ? 32 : 64;
  }
  // pair: 0 one CTA per tile, 1 a CTA pair (2-SM UMMA), 2 one CTA per tile with the k split, 3 a CTA pair with
  // the k split
  const int cg = pair == 1 || pair == 3 ? 2 : 1;
  if (cg == 2 && bn != 128) bn = 256;  // the pair tiles are 256 x 256 and 256 x 128
  const int b_mn = g->opB == 1, a_mn = g->opA == 0;
  if (b_mn && bn / cg < epr) bn = epr * cg;  // an MN-major B tile holds whole 128-byte rows
  const int b_rows = bn / cg;
  const CUtensorMapDataType dt =
      f32in ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
            : (g->in_type == TB200_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);

  TcParams p;
  memset(&p, 0, sizeof p);
  CUtensorMap ta, tb;
  bool ok;
  // the 256 x 256 pair tile: one 64-deep k-chunk per stage (six stages), or two (three stages: half the MMA
  // thread's barrier waits and commits per k) for launches of at least three waves. Measured on the B200 against
  // one chunk, bit-identical results: lm_head 128256 x 512 x 4096 1-1.5 % and 8192^3 4-6 % faster, gate 14336 x
  // 512 x 4096 (1.5 waves) 2 % slower.
  const char *ks_env = getenv("TB200_KSPLIT");
  const long long pair_tiles = (long long)((g->m + 255) / 256) * ((g->n + 255) / 256) * (g->batch > 0 ? g->batch : 1);
  const bool pair_kc2 = cg == 2 && bn == 256 && pair == 1 && !f32in && !g->gidx && !(ks_env && *ks_env == '1') &&
                        pair_tiles >= 3LL * (num_sms / 2);
  const int kc = cg == 2 && bn == 256 ? (pair_kc2 ? 2 : 1) : kc_for(bn);
  // pointer arrays: rank-2 template maps with a placeholder address, re-pointed per element on the device
  const void *baseA = ptr_ws ? (const void *)(uintptr_t)0x10000 : g->A;
  const void *baseB = ptr_ws ? (const void *)(uintptr_t)0x10000 : g->B;
  const int mbatch = ptr_ws ? 1 : g->batch;
  if (!a_mn) ok = make_map(&ta, dt, es, baseA, g->k, g->m, g->lda, mbatch, g->sA, epr, TC_BM, &p.a_batched);
  else ok = make_map(&ta, dt, es, baseA, g->m, g->k, g->lda, mbatch, g->sA, epr, epr * kc, &p.a_batched);
  if (ok && g->gidx) {
    ok = make_map(&tb, dt, es, g->B, g->k, g->n_src, g->ldb, 1, 0, epr, 1, &p.b_batched);  // box one column
  } else if (ok) {
    if (!b_mn) ok = make_map(&tb, dt, es, baseB, g->k, g->n, g->ldb, mbatch, g->sB, epr, b_rows, &p.b_batched);
    else ok = make_map(&tb, dt, es, baseB, g->n, g->k, g->ldb, mbatch, g->sB, epr, epr * kc, &p.b_batched);
  }
  if (!ok && ptr_ws) return (int)cudaErrorNotSupported;  // the caller takes the general kernel
  if (!ok) {
    if (g->nrep || g->mc || g->groups) return (int)cudaErrorNotSupported;  // tensor-core only
    if (tb200_trace()) fprintf(stderr, "[trace] tensor map refused; SIMT kernel instead\n");
    return tb200_launch_simt(g, s);
  }
  p.m = g->m; p.n = g->n; p.k = g->k; p.batch = g->batch;
  p.epr = epr;
  p.bk = epr * kc;
  p.num_kb = (g->k + p.bk - 1) / p.bk;
  p.m_tiles = (g->m + TC_BM * cg - 1) / (TC_BM * cg);
  p.n_tiles = (g->n + bn - 1) / bn;
  p.tiles_per_batch = (long long)p.m_tiles * p.n_tiles;
  p.total_tiles = p.tiles_per_batch * g->batch;
  p.group_m = 8;
  p.alpha = g->alpha; p.beta = g->beta;
  p.C = g->C; p.ldc = g->ldc; p.sC = g->sC; p.out_type = g->out_type;
  p.nrep = g->nrep;
  p.row0 = g->row0;
  p.mc = (float *)g->mc;
  // grouped GEMM: the tile count is known only on the device; total_tiles (m-tiles x n-tiles over all columns,
  // per group) bounds it and sizes the grid
  p.groups = g->groups;
  p.grp_off = g->grp_off;
  p.gidx = g->gidx;
  p.n_src = g->n_src;
  for (int q = 0; q < g->nrep && q < 8; ++q) p.rep[q] = g->rep[q];
  if (ptr_ws) {
    int *flag = (int *)ptr_ws;
    CUtensorMap *maps = (CUtensorMap *)((char *)ptr_ws + 256);
    p.maps = maps;
    p.Carr = g->Carr;
    p.skip = flag;
    // this call's number (never 0, the value of a fresh, zeroed flag): a flag raised by an earlier call on the same
    // scratch does not match it
    static unsigned next_gen;
    unsigned gen = __atomic_add_fetch(&next_gen, 1u, __ATOMIC_RELAXED) & 0x7fffffffu;
    if (gen == 0) gen = __atomic_add_fetch(&next_gen, 1u, __ATOMIC_RELAXED) & 0x7fffffffu;
    p.skip_gen = (int)gen;
    g_last_ptr_gen = (int)gen;
    cudaError_t e;
    const unsigned blocks = (unsigned)((g->batch + 127) / 128);
    if (tb200_trace())
      fprintf(stderr, "[trace] launch tb200_ptr_maps_kernel grid=(%u,1,1) block=(128,1,1) batch=%d\n", blocks, g->batch);
    cudaLaunchConfig_t pcfg = {};
    cudaLaunchAttribute pat[1];
    pat[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pat[0].val.programmaticStreamSerializationAllowed = 1;
    pcfg.gridDim = dim3(blocks, 1, 1);
    pcfg.blockDim = dim3(128, 1, 1);
    pcfg.stream = s;
    pcfg.attrs = pat;
    pcfg.numAttrs = tb200_pdl() ? 1 : 0;
    e = cudaLaunchKernelEx(&pcfg, tb200_ptr_maps_kernel, ta, tb, g->Aarr, g->Barr, maps, g->batch, flag, p.skip_gen);
    if (e != cudaSuccess) return (int)e;
  }
  // the TMA-store epilogue, where C is this GPU's own plain C with beta == 0 and its base and leading dimension
  // suit a tensor map (16-byte multiples). Strided batches keep the per-lane stores: measured on the B200 (three
  // rounds, one box), config 3's KQ and KQV ran 1.5-2 % faster with them, while lm_head ran 1.5 % faster with
  // the TMA stores. TB200_TMA_STORE=0 never, =1 strided batches too (tests, bisecting; read per call)
  CUtensorMap tcm;
  memset(&tcm, 0, sizeof tcm);
  {
    const char *e = getenv("TB200_TMA_STORE");
    const int esc = g->out_type == TB200_F32 ? 4 : 2;
    const bool batched_ok = e && *e == '1' && g->sC > 0 && (g->sC * esc) % 16 == 0;
    if (!(e && *e == '0') && !ptr_ws && !g->nrep && !g->mc && !g->groups && !g->gidx && g->beta == 0.f && g->C &&
        ((uintptr_t)g->C & 15) == 0 && ((long long)g->ldc * esc) % 16 == 0 && (g->batch == 1 || batched_ok))
      p.c_tma = make_c_map(&tcm, g->out_type, g->C, g->m, g->n, g->ldc, g->batch, g->sC, &p.c_batched) ? 1 : 0;
    // plain f32 per-lane stores drain TMEM in 16-column halves, the next half's load in flight while this half's
    // stores issue: config 3's KQ 58.6-58.9 -> 57.1-57.3 us, KQV ~0.5 %, bit-identical C (same-process A/B, three
    // rounds). TB200_EPI_PIPE=0 keeps the 32-column loop (bisecting; read per call)
    const char *pipe = getenv("TB200_EPI_PIPE");
    p.epi_pipe = !(pipe && *pipe == '0');
  }
  // TB200_WAIT_BUDGET_CYC shortens the pipeline waits' budget (tests; read per call); the drain waits after an
  // abort keep theirs. TB200_TEST_STALL=1 plants the MMA thread's wait that nothing completes (tests only).
  {
    const char *e = getenv("TB200_WAIT_BUDGET_CYC");
    const long long v = e && *e ? atoll(e) : 0;
    p.wait_budget = v > 0 && (uint64_t)v < WAIT_BUDGET_CYC ? (uint64_t)v : WAIT_BUDGET_CYC;
    const char *st = getenv("TB200_TEST_STALL");
    p.test_stall = st && *st == '1';
  }
  p.a_mn = a_mn; p.b_mn = b_mn;
  // K-major: 8-row core groups 1024 bytes apart (SBO), chunk c of a stage rows*128 bytes in, UMMA_K step
  // = 32 bytes inside the swizzle atom. MN-major: 128-byte rows along m/n, 8 k-rows per 1024-byte atom
  // (SBO), atoms along m/n one box (bk rows x 128 bytes) apart (LBO), UMMA_K step = UMMA_K rows of 128
  // bytes, and a stage's chunks follow each other inside the box.
  const uint32_t umma_k = 32 / es;
  p.a_lbo = a_mn ? (uint32_t)(p.bk * 128) : 16u;
  p.a_sbo = 1024u;
  p.a_kstep = a_mn ? umma_k * 128u : 32u;
  p.a_cstride = a_mn ? 4u * p.a_kstep : (uint32_t)(TC_BM * 128);
  p.b_lbo = b_mn ? (uint32_t)(p.bk * 128) : 16u;
  p.b_sbo = 1024u;
  p.b_kstep = b_mn ? umma_k * 128u : 32u;
  p.b_cstride = b_mn ? 4u * p.b_kstep : (uint32_t)(b_rows * 128);
  const uint32_t fmt = f32in ? 2u : (g->in_type == TB200_BF16 ? 1u : 0u);
  p.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
            ((uint32_t)(bn >> 3) << 17) | ((uint32_t)((TC_BM * cg) >> 4) << 24);

  // the k split (KS = 2, the planner's modes 2 and 3): two halves of a cluster per tile (two CTAs, or two CTA
  // pairs), one tile per cluster, each half with half the k-blocks, for 16-bit GEMMs whose tiles leave at
  // least half of the SMs idle. TB200_KSPLIT=0 never, =1 whenever allowed, whatever the planner chose (tests,
  // bisecting; read per call).
  int rc = (int)cudaErrorNotSupported;
  {
    const char *e = getenv("TB200_KSPLIT");
    const int want = e && *e ? atoi(e) : -1;
    const bool allowed = !f32in && !ptr_ws && !g->groups && !g->nrep && !g->mc && p.num_kb >= 2 &&
                         (cg == 2 ? bn == 256 : bn == 64 || bn == 128 || bn == 256) &&
                         p.total_tiles * 2 * cg <= num_sms && (pair >= 2 || want == 1);
    if (allowed && want != 0 && cg == 2) {
      rc = launch_bn<0, 256, 1, 2, 2>(ta, tb, tcm, p, num_sms, s);
    } else if (allowed && want != 0) {
      switch (bn) {
        case 64: rc = launch_bn<0, 64, kc_for(64), 1, 2>(ta, tb, tcm, p, num_sms, s); break;
        case 128: rc = launch_bn<0, 128, kc_for(128), 1, 2>(ta, tb, tcm, p, num_sms, s); break;
        default: rc = launch_bn<0, 256, kc_for(256), 1, 2>(ta, tb, tcm, p, num_sms, s); break;
      }
    }
  }
  if (rc != (int)cudaErrorNotSupported) {
    // launched (or failed) with the k split
  } else if (cg == 2) {
    if (bn == 128)
      rc = f32in ? launch_bn<1, 128, 2, 2>(ta, tb, tcm, p, num_sms, s) : launch_bn<0, 128, 2, 2>(ta, tb, tcm, p, num_sms, s);
    else
      rc = f32in      ? launch_bn<1, 256, 1, 2>(ta, tb, tcm, p, num_sms, s)
           : pair_kc2 ? launch_bn<0, 256, 2, 2>(ta, tb, tcm, p, num_sms, s)
                      : launch_bn<0, 256, 1, 2>(ta, tb, tcm, p, num_sms, s);
  } else if (f32in) {
    switch (bn) {
      case 32: rc = launch_bn<1, 32, kc_for(32), 1>(ta, tb, tcm, p, num_sms, s); break;
      case 64: rc = launch_bn<1, 64, kc_for(64), 1>(ta, tb, tcm, p, num_sms, s); break;
      case 128: rc = launch_bn<1, 128, kc_for(128), 1>(ta, tb, tcm, p, num_sms, s); break;
      default: rc = launch_bn<1, 256, kc_for(256), 1>(ta, tb, tcm, p, num_sms, s); break;
    }
  } else {
    switch (bn) {
      case 32: rc = launch_bn<0, 32, kc_for(32), 1>(ta, tb, tcm, p, num_sms, s); break;
      case 64: rc = launch_bn<0, 64, kc_for(64), 1>(ta, tb, tcm, p, num_sms, s); break;
      case 128: rc = launch_bn<0, 128, kc_for(128), 1>(ta, tb, tcm, p, num_sms, s); break;
      default: rc = launch_bn<0, 256, kc_for(256), 1>(ta, tb, tcm, p, num_sms, s); break;
    }
  }
  if (rc != 0 || !ptr_ws) return rc;
  // the general kernel behind it: it computes the batch only if some pointer was unfit for TMA
  tb200_gemm_t gf = *g;
  gf.run_if = p.skip;
  gf.run_if_gen = p.skip_gen;
  return tb200_launch_simt(&gf, s);
}

extern "C" int tb200_launch_tc(const tb200_gemm_t *g, int tile_n, int pair, int num_sms, cudaStream_t s) {
  // only the tensor-core epilogue replicates rows, and only this kernel runs grouped GEMMs
  if (!tb200_tc_ok(g))
    return (g->nrep || g->mc || g->groups) ? (int)cudaErrorNotSupported : tb200_launch_simt(g, s);
  return launch_tc_impl(g, tile_n, pair, num_sms, nullptr, s);
}

extern "C" size_t tb200_tc_ptr_ws_bytes(int batch) { return 256 + (size_t)(batch > 0 ? batch : 0) * 256; }

extern "C" int tb200_launch_tc_ptr(const tb200_gemm_t *g, int tile_n, int pair, int num_sms, void *ws, cudaStream_t s) {
  const int es = g->in_type == TB200_F32 ? 4 : 2;
  if (!ws || !g->Aarr || !g->Barr || !g->Carr || g->nrep || g->k <= 0) return (int)cudaErrorNotSupported;
  if (g->in_type == TB200_F32 && (g->opA != 1 || g->opB != 0)) return (int)cudaErrorNotSupported;
  if (((long long)g->lda * es) % 16 || ((long long)g->ldb * es) % 16) return (int)cudaErrorNotSupported;
  if (((uintptr_t)ws) & 255) return (int)cudaErrorNotSupported;
  return launch_tc_impl(g, tile_n, pair, num_sms, ws, s);
}

extern "C" __attribute__((visibility("default"))) int tb200_device_error(void) {
  int v = 0, zero = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, g_tb200_err, sizeof v) != cudaSuccess) return -1;
  cudaMemcpyToSymbol(g_tb200_err, &zero, sizeof zero);
  return v;
}

// ---------------------------------------------------------------------------------------------------
// Allocation-free variant of the pointer-array launch.
//
// The pointer-array path needs device scratch for one pair of tensor maps per batch element (plus a flag).
// tb200_gemm_batched_ex_noalloc serves callers that must not have the library call cudaMalloc: their
// scratch is this fixed array, part of the library's device image, so every GPU that loads the library
// holds its 256 KB + 256 B until the process exits. It bounds the batch at TB200_NOALLOC_MAX_BATCH.
// All calls, on every stream, share it and it keeps the last call's contents: the flag starts at zero (the
// array is zero when the library is loaded) and is never cleared - each call compares it with its own
// generation number - the maps are rewritten for every element, and calls whose launches overlap on the GPU
// race on it.
#define TB200_NOALLOC_MAX_BATCH 1024
static __device__ __align__(256) unsigned char g_tb200_noalloc_scratch[256 + TB200_NOALLOC_MAX_BATCH * 256];

// The host-side name g_tb200_noalloc_scratch is only a stand-in for the symbol, never a device address:
// the device address comes from cudaGetSymbolAddress, looked up with the device current. The first call on
// each of the first 64 device ordinals caches it (an atomic store, so concurrent first calls agree); higher
// ordinals look it up on every call. The cache is not rebuilt after cudaDeviceReset, which unloads the
// library's device image: a process that resets a device must not call this entry point on it afterwards.
static void *noalloc_scratch(void) {
  static void *addr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return nullptr;
  void *cached = dev < 64 ? __atomic_load_n(&addr[dev], __ATOMIC_ACQUIRE) : nullptr;
  if (cached) return cached;
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_tb200_noalloc_scratch);
  if (e != cudaSuccess || !p) {
    fprintf(stderr, "[tinycublas_b200] cudaGetSymbolAddress(scratch) failed on device %d: %s\n", dev,
            cudaGetErrorString(e));
    (void)cudaGetLastError();
    return nullptr;
  }
  if (dev < 64) __atomic_store_n(&addr[dev], p, __ATOMIC_RELEASE);
  return p;
}

// Test hook: 1 when the last allocation-free call on the current device found some batch pointer unfit for
// TMA (the general kernel then ran the batch), 0 when its tensor-core launch ran, -1 on error. Waits for the
// device.
static int g_noalloc_last_gen;  // generation number of the last allocation-free pointer-array launch

extern "C" __attribute__((visibility("default"))) int tb200_noalloc_last_fallback(void) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, g_tb200_noalloc_scratch, sizeof v) != cudaSuccess) return -1;
  return g_noalloc_last_gen != 0 && v == g_noalloc_last_gen ? 1 : 0;
}

extern "C" __attribute__((visibility("default"))) int tb200_noalloc_max_batch(void) { return TB200_NOALLOC_MAX_BATCH; }

extern "C" int tb200_launch_tc_ptr_noalloc(const tb200_gemm_t *g, int tile_n, int pair, int num_sms, cudaStream_t s) {
  if (g->batch > TB200_NOALLOC_MAX_BATCH || tb200_tc_ptr_ws_bytes(g->batch) > sizeof(g_tb200_noalloc_scratch))
    return (int)cudaErrorInvalidValue;
  void *ws = noalloc_scratch();
  if (!ws) return (int)cudaErrorInvalidSymbol;
  const int rc = tb200_launch_tc_ptr(g, tile_n, pair, num_sms, ws, s);
  g_noalloc_last_gen = g_last_ptr_gen;
  return rc;
}
