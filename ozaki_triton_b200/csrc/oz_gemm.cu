// oz_gemm.cu -- fused Ozaki cross-GEMM on the 5th-generation tensor cores
// (tcgen05, sm_100a).
//
// Replaces cross_gemm_kernel (ozaki_triton.py:305-452) and its wrapper
// cross_gemm (ozaki_triton.py:455-498):
//   C[b,m,n] = out( sum_i sum_j od( f32( f32(acc_ij[m,n]) * sa_i[m] ) * sb_j[n] ) )
//   acc_ij   = sum_k A_i[m,k] * B_j[n,k]   (int32 for int8 slices, fp32 otherwise)
// summed i-major, j-minor into od = fp64 (fp64 output) or fp32, exactly the
// epilogue order of ozaki_triton.py:426-447, so int8 results are bit-identical
// to the reference.
//
// Structure (one persistent CTA per SM, 10 warps):
//   warp 0     TMA producer: per 128-byte K block, the A_i tile and the
//              stacked tiles of all B_j (one 3-D box) into one ring stage.
//   warp 1     TMEM allocator + single-thread tcgen05.mma issuer.
//   warps 2-9  epilogue: the tile's B scales staged once in shared memory,
//              tcgen05.ld of the int32/fp32 accumulators, scaling, fp64/fp32
//              outer accumulation in registers, store of C.
// Per output tile (128 rows x NT columns) the kernel runs one "pass" per A
// slice i, or per two A slices when their 2 * s accumulators fit TMEM: a full
// K loop that accumulates the pair products A_i B_j for every j into s TMEM
// accumulators of NT columns each (pa * s * NT <= 512 columns).  A_i is
// loaded once per pass and reused by all j, and B's stack once per pass for
// its pa A slices; when 2 * pa * s * NT <= 512 the accumulators are
// double-buffered so the epilogue of one pass overlaps the MMAs of the next.
// The fp64/fp32 outer accumulator never leaves registers.
//
// Every spin-wait is bounded (oz_common.cuh); on a timeout the kernel records
// a code in g_device_status, drains its own asynchronous work (bounded), frees
// TMEM and returns.

#include <cstdio>
#include <cstdlib>
#include <cudaTypedefs.h>

#include "oz_common.cuh"
#include "oz_tile_table.h"

namespace oz {

constexpr int kBM = 128;          // rows per CTA (UMMA M per CTA)
constexpr int kKBytes = 128;      // K bytes per pipeline stage (one swizzle row)
constexpr int kGemmThreads = 320; // 10 warps
constexpr int kEpiWarps = 8;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 225 * 1024;   // stages + alignment slack
constexpr int kBarrierBytes = 1024;

struct GemmParams {
  const float *a_scales;
  const float *b_scales;
  const int32_t *a_index;
  const int32_t *b_index;
  void *c;
  int64_t ldc;
  int m, n, kblocks;     // kblocks = ld_bytes / 128
  int s;
  int skip_tail;
  int batch;
  int tiles_m, tiles_n, num_tiles;
  int gm;                // row tiles per raster group
  int bw, bblocks;       // B stored in column blocks of bw columns (bblocks per batch)
  int stages;            // pipeline depth
  int pa;                // A slices per pass (1, or 2 when 2 * s * NT fits the 512 TMEM columns)
  uint32_t idesc;        // instruction descriptor without the N field
  // column blocks still arriving (oz_cross_gemm_arrivals; ready == nullptr:
  // every block present): the tiles of block_count blocks go block by block
  // from first_block on, and block c is read once ready[c] == ready_value
  const int *ready;
  int ready_value;
  int first_block;
  int tiles_bn;          // column tiles per column block
};

// One pipeline stage holds, for one 128-byte K block, the A tiles of the
// pass (128 rows of each of its pa A slices) followed by the stacked B tiles
// of all s slices (s x NT/PAIR rows: B_0 rows, B_1 rows, ...).  Stacking lets
// one MMA with N = 256 cover several slices at once: its accumulator columns
// are the products with consecutive B slices.  Two A slices per pass (when
// their 2 * s accumulators fit TMEM) double the MMA work per fed byte of B.
__host__ __device__ constexpr int a_tile_bytes() { return kBM * kKBytes; }
__host__ __device__ inline int stage_bytes(int s, int nt, int pair, int pa) {
  return pa * a_tile_bytes() + s * (nt / pair) * kKBytes;
}

// B scales of a tile staged for the epilogue: two tiles x s slices x NT floats.
__host__ __device__ inline int scale_stage_bytes(int s, int nt) { return 2 * s * nt * 4; }

template <int OUTK> struct OutT;
template <> struct OutT<OZ_F64> { using acc = double; using store = double; };
template <> struct OutT<OZ_F32> { using acc = float; using store = float; };
template <> struct OutT<OZ_F16> { using acc = float; using store = __half; };
template <> struct OutT<OZ_BF16> { using acc = float; using store = __nv_bfloat16; };
template <> struct OutT<OZ_I8> { using acc = float; using store = int8_t; };

template <typename ACC> __device__ __forceinline__ ACC acc_add(ACC a, float v);
template <> __device__ __forceinline__ double acc_add<double>(double a, float v) {
  return __dadd_rn(a, (double)v);
}
template <> __device__ __forceinline__ float acc_add<float>(float a, float v) {
  return __fadd_rn(a, v);
}

template <int OUTK> __device__ __forceinline__ typename OutT<OUTK>::store
to_out(typename OutT<OUTK>::acc v) {
  if constexpr (OUTK == OZ_F16) return __float2half_rn(v);
  else if constexpr (OUTK == OZ_BF16) return __float2bfloat16_rn(v);
  else if constexpr (OUTK == OZ_I8) {
    // int8 inputs give an int8 result: truncation toward zero, saturated to
    // [-128, 127], NaN -> 0 (the GPU's float-to-int8 conversion)
    return (int8_t)max(-128, min(127, __float2int_rz(v)));
  } else return v;
}

// tile t -> (batch b, row tile mb, column tile nb) in a grouped raster:
// GM row tiles sweep all column tiles before moving on, so the A rows and B
// columns of the tiles running at the same time stay in L2.  With arriving
// column blocks the tiles go block by block in arrival order (first_block,
// first_block + 1, .. modulo the number of blocks, one batch), the same
// raster inside each block; blk is the tile's column block.  Returns false
// for a tile past the last column (a short last block), which every role
// skips.
__device__ __forceinline__ bool tile_coords(const GemmParams &p, int t, int &b, int &mb, int &nb,
                                            int &blk) {
  const int GM = p.gm;
  int local, cols, nb0 = 0;
  if (p.ready) {
    const int tpb = p.tiles_m * p.tiles_bn;
    const int ord = t / tpb;
    b = 0;
    local = t - ord * tpb;
    blk = (p.first_block + ord) % p.bblocks;
    cols = p.tiles_bn;
    nb0 = blk * p.tiles_bn;
  } else {
    const int tpb = p.tiles_m * p.tiles_n;
    b = t / tpb;
    local = t - b * tpb;
    cols = p.tiles_n;
  }
  int per_group = GM * cols;
  int group = local / per_group;
  int first_m = group * GM;
  int gsz = min(p.tiles_m - first_m, GM);
  int in_group = local - group * per_group;
  mb = first_m + in_group % gsz;
  nb = nb0 + in_group / gsz;
  if (!p.ready) blk = 0;
  return nb < p.tiles_n;
}

// Bounded wait for a column block's arrival flag (acquire, then ordered
// before the async proxy's TMA reads of the block).  The flag is written by
// a copy engine, which needs no SM, so waiting here cannot starve the writer.
__device__ __forceinline__ bool wait_block(const GemmParams &p, int blk, uint64_t &seen,
                                           volatile int *abort_flag) {
  if (!p.ready || (blk < 64 && ((seen >> blk) & 1))) return true;
  const int *f = p.ready + blk;
  const long long t0 = clock64();
  for (;;) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v == p.ready_value) break;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitBoundCycles) {
      *abort_flag = DEV_TIMEOUT_ARRIVAL;
      atomicCAS(&g_device_status, 0, (int)DEV_TIMEOUT_ARRIVAL);
      return false;
    }
    __nanosleep(200);
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  if (blk < 64) seen |= 1ull << blk;
  return true;
}

// PAIR == 1: one CTA computes a 128 x NT tile with cta_group::1 MMAs.
// PAIR == 2: a cluster of two CTAs computes a 256 x NT tile; each CTA loads
//            its 128 A rows and NT/2 rows of every B slice, the leader
//            (rank 0) issues cta_group::2 MMAs over both CTAs' shared memory
//            and each CTA's TMEM receives its own 128 rows.  Loads of both
//            CTAs complete on the leader's "full" barriers; the leader's
//            commits release the "empty" barriers and signal the
//            accumulators of both CTAs.
// TMEM layout of one pass: group g of up to 256 columns holds the products
// with slices [g*SPG, g*SPG + SPG) (SPG = 256 / NT).  PAIR == 1: column
// g*256 + jj*NT + x is slice g*SPG+jj, tile column x.  PAIR == 2: the first
// Rg columns of a group come from the leader's B rows (tile columns
// [0, NT/2)), the next Rg from the peer's (tile columns [NT/2, NT)), with
// Rg = NT/2 * (slices in the group).
// 320 threads: registers are split per SM sub-partition (16K each, up to 3
// warps on one), so a thread gets at most 168 -- 128 of them hold the
// epilogue's 64 fp64 accumulators.
template <int KIND, int OUTK, int NT, int PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    cross_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                      const __grid_constant__ CUtensorMap tm_b, const GemmParams p) {
  using ACC = typename OutT<OUTK>::acc;
  using STO = typename OutT<OUTK>::store;
  constexpr int TM = kBM * PAIR;                  // rows of one tile
  constexpr int R = NT / PAIR;                    // B rows per slice held by one CTA
  constexpr int SPG = 256 / NT;                   // slices per MMA group
  constexpr int NH = NT / 2;                      // tile columns per epilogue warp half

  const int s = p.s;
  const int S = p.stages;
  const int PA = p.pa;
  const int sbytes = stage_bytes(s, NT, PAIR, PA);
  const int bofs = PA * a_tile_bytes();          // B stack offset inside a stage
  const int pcols = PA * s * NT;                  // TMEM columns of one pass

  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char *smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S * sbytes);
  uint64_t *full = bars;                  // [S]
  uint64_t *empty = full + kMaxStages;    // [S]
  uint64_t *acc_full = empty + kMaxStages;  // [2]
  uint64_t *acc_empty = acc_full + 2;     // [2]
  uint64_t *drain = acc_empty + 2;        // [1]
  uint64_t *sb_ready = drain + 1;         // [2] B scales of a tile staged
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sb_ready + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int nbuf = (2 * pcols <= 512) ? 2 : 1;
  int tcols = 32;
  while (tcols < nbuf * pcols) tcols <<= 1;
  const uint32_t rank = (PAIR == 2) ? cluster_ctarank() : 0;
  const bool leader = rank == 0;
  const int unit = blockIdx.x / PAIR;          // this CTA's pair (or CTA) index
  const int units = gridDim.x / PAIR;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], PAIR * kEpiWarps * 32);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&sb_ready[i], kEpiWarps * 32);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
  }
  if (warp == 1) {
    if constexpr (PAIR == 2) {
      tmem_alloc_pair(tmem_slot, (uint32_t)tcols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, (uint32_t)tcols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR == 2) cluster_sync();   // barriers of both CTAs initialised
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // shared::cluster address of a barrier in the leader CTA
  auto leader_addr = [&](uint64_t *bar) -> uint32_t {
    if constexpr (PAIR == 2) return map_to_cta(smem_u32(bar), 0);
    else return smem_u32(bar);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;           // running stage counter (slot = it % S)
      bool ok = true;
      const uint32_t tx = (uint32_t)(PAIR * sbytes);
      uint64_t seen = 0;         // column blocks known to have arrived
      for (int t = unit; ok && t < p.num_tiles; t += units) {
        int b, mb, nb, ablk;
        if (!tile_coords(p, t, b, mb, nb, ablk)) continue;
        if (!(ok = wait_block(p, ablk, seen, abort_flag))) break;
        const int ai = p.a_index ? p.a_index[b] : b;
        const int bi = p.b_index ? p.b_index[b] : b;
        const int arow = mb * TM + (int)rank * kBM;
        // B column blocks: a tile never straddles two (bw is a multiple of NT)
        const int blk = (nb * NT) / p.bw;
        const int brow = nb * NT - blk * p.bw + (int)rank * R;
        const int bz = (bi * p.bblocks + blk) * s;
        for (int i = 0; ok && i < s; i += PA) {
          for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
            const int slot = it % S;
            if (!(ok = mbar_wait_bounded(&empty[slot], ((it / S) & 1) ^ 1, abort_flag,
                                         DEV_TIMEOUT_PRODUCER)))
              break;
            unsigned char *st = smem + slot * sbytes;
            if constexpr (PAIR == 2) {
              if (leader) mbar_arrive_expect_tx(&full[slot], tx);
              const uint32_t fb = leader_addr(&full[slot]);
              tma_load_3d_pair(st, &tm_a, fb, kb * kKBytes, arow, ai * s + i);   // PA slices
              tma_load_3d_pair(st + bofs, &tm_b, fb, kb * kKBytes, brow, bz);
            } else {
              mbar_arrive_expect_tx(&full[slot], tx);
              tma_load_3d(st, &tm_a, &full[slot], kb * kKBytes, arow, ai * s + i);   // PA slices
              tma_load_3d(st + bofs, &tm_b, &full[slot], kb * kKBytes, brow, bz);
            }
          }
        }
      }
      // drain: every load the leader's barriers count must have landed
      // before shared memory is released
      if (leader)
        for (uint32_t k = (it > (uint32_t)S ? it - S : 0); k < it; ++k)
          mbar_wait_bounded(&full[k % S], (k / S) & 1, abort_flag, DEV_TIMEOUT_PRODUCER);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      uint32_t it = 0, pass = 0;
      bool ok = true;
      const uint32_t base = smem_u32(smem);
      auto release = [&](uint64_t *bar) {
        if constexpr (PAIR == 2) {
          tc_commit_pair(smem_u32(bar));                     // own barrier
          tc_commit_pair(map_to_cta(smem_u32(bar), 1));      // the peer's barrier
        } else {
          tc_commit(bar);
        }
      };
      for (int t = unit; ok && t < p.num_tiles; t += units) {
        int b_, mb_, nb_, blk_;
        if (!tile_coords(p, t, b_, mb_, nb_, blk_)) continue;
        for (int i = 0; ok && i < s; i += PA, ++pass) {
          const int buf = pass % nbuf;
          const uint32_t use = pass / nbuf;
          if (!(ok = mbar_wait_bounded(&acc_empty[buf], (use & 1) ^ 1, abort_flag,
                                       DEV_TIMEOUT_MMA)))
            break;
          tc_fence_after();
          const uint32_t d0 = tmem_base + (uint32_t)(buf * pcols);
          for (int kb = 0; kb < p.kblocks; ++kb, ++it) {
            const int slot = it % S;
            if (!(ok = mbar_wait_bounded(&full[slot], (it / S) & 1, abort_flag, DEV_TIMEOUT_MMA)))
              break;
            const uint32_t sa = base + slot * sbytes;
            const int pc = min(PA, s - i);             // A slices in this pass
#pragma unroll 1
            for (int a = 0; a < pc; ++a) {
              // A slice i + a: its accumulators follow those of slice i
              const int js = p.skip_tail ? s - (i + a) : s;
              const int groups = (js + SPG - 1) / SPG;
              const uint64_t adesc = smem_desc_sw128(sa + a * a_tile_bytes());
              const uint32_t da = d0 + (uint32_t)(a * s * NT);
#pragma unroll 1
              for (int g = 0; g < groups; ++g) {
                const int sg = min(SPG, js - g * SPG);
                const uint32_t idesc = p.idesc | ((uint32_t)((sg * NT) >> 3) << 17);
                const uint64_t bdesc = smem_desc_sw128(sa + bofs + g * (256 / PAIR) * kKBytes);
#pragma unroll
                for (int kk = 0; kk < kKBytes / 32; ++kk) {
                  // advance 32 bytes along K inside the 128-byte swizzle row
                  if constexpr (PAIR == 2)
                    tc_mma_pair<KIND>(da + (uint32_t)(g * 256), adesc + (uint64_t)(kk * 2),
                                      bdesc + (uint64_t)(kk * 2), idesc, (kb | kk) != 0);
                  else
                    tc_mma<KIND>(da + (uint32_t)(g * 256), adesc + (uint64_t)(kk * 2),
                                 bdesc + (uint64_t)(kk * 2), idesc, (kb | kk) != 0);
                }
              }
            }
            release(&empty[slot]);
          }
          if (!ok) break;
          release(&acc_full[buf]);
        }
      }
      // wait for all issued MMAs before TMEM / shared memory go away
      if constexpr (PAIR == 2) tc_commit_pair(smem_u32(drain));
      else tc_commit(drain);
      mbar_wait_bounded(drain, 0, abort_flag, DEV_TIMEOUT_MMA);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 2;
    const int sub = warp & 3;                 // TMEM lane quarter this warp may access
    const int half = e >> 2;                  // which half of the NT tile columns
    const int et = threadIdx.x - 64;          // epilogue thread 0..255
    const int row = (int)rank * kBM + sub * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(sub * 32) << 16);
    const uint32_t empty_addr0 = leader_addr(&acc_empty[0]);
    const uint32_t empty_addr1 = leader_addr(&acc_empty[1]);
    // B scales of the current tile, [2 tiles][s][NT], read as warp-wide broadcasts
    float *sb_stage = reinterpret_cast<float *>(smem + S * sbytes + kBarrierBytes);
    ACC out[NH];
#pragma unroll
    for (int x = 0; x < NH; ++x) out[x] = (ACC)0;
    uint32_t pass = 0;
    int tile_iter = -1;                       // tiles of this CTA processed, minus one
    bool ok = true;
    uint64_t seen = 0;                        // column blocks known to have arrived
    for (int t = unit; ok && t < p.num_tiles; t += units) {
      int b, mb, nb, ablk;
      if (!tile_coords(p, t, b, mb, nb, ablk)) continue;
      ++tile_iter;
      // the B scales of an arriving block are read only once it is here
      ok = __all_sync(0xffffffffu, wait_block(p, ablk, seen, abort_flag));
      if (!ok) break;
      const int ai = p.a_index ? p.a_index[b] : b;
      const int bi = p.b_index ? p.b_index[b] : b;
      const int m = mb * TM + row;
      const int n0 = nb * NT + half * NH;
      const int blk = (nb * NT) / p.bw;
      // stage the tile's B scales; a warp passes the staging barrier of tile
      // t + 1 only when every epilogue warp has finished tile t, so the
      // buffer of tile t + 2 is free when it is written
      float *sbt = sb_stage + (tile_iter & 1) * s * NT;
      {
        const float *src = p.b_scales + ((int64_t)bi * p.bblocks + blk) * s * p.bw;
        const int c0 = nb * NT - blk * p.bw;   // first tile column inside its block
        for (int q = et; q < s * NT; q += kEpiWarps * 32) {
          const int j = q / NT, x = q - j * NT;
          sbt[q] = (nb * NT + x < p.n) ? __ldg(src + (int64_t)j * p.bw + c0 + x) : 0.f;
        }
      }
      mbar_arrive(&sb_ready[tile_iter & 1]);
      ok = mbar_wait_bounded(&sb_ready[tile_iter & 1], (tile_iter >> 1) & 1, abort_flag,
                             DEV_TIMEOUT_EPILOGUE);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      for (int i = 0; i < s; i += PA, ++pass) {
        const int buf = pass % nbuf;
        const uint32_t use = pass / nbuf;
        // every lane waits, then the warp agrees (tcgen05.ld needs a converged warp)
        ok = mbar_wait_bounded(&acc_full[buf], use & 1, abort_flag, DEV_TIMEOUT_EPILOGUE);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        // A slices i, i + 1, .. of the pass in order, each with its B slices
        // in order: the reference's i-major, j-minor sum
        const int pc = min(PA, s - i);
        for (int a = 0; a < pc; ++a) {
          const int ia = i + a;
          const int js = p.skip_tail ? s - ia : s;
          const float sa = (m < p.m) ? p.a_scales[((int64_t)ai * s + ia) * p.m + m] : 0.f;
          for (int j = 0; j < js; ++j) {
            const float *sbj = sbt + j * NT + half * NH;
            const int g = j / SPG, jj = j % SPG;
            int col;
            if constexpr (PAIR == 2) {
              const int rg = min(SPG, js - g * SPG) * NH;    // columns per CTA half in group
              col = buf * pcols + a * s * NT + g * 256 + half * rg + jj * NH;
            } else {
              col = buf * pcols + a * s * NT + g * 256 + jj * NT + half * NH;
            }
#pragma unroll
            for (int c = 0; c < NH / 16; ++c) {
              uint32_t r[16];
              tmem_ld16_at(lane_addr + (uint32_t)(col + c * 16), r);
              tmem_ld_wait16(r);
#pragma unroll
              for (int x = 0; x < 16; ++x) {
                const float sb = sbj[c * 16 + x];
                float v;
                if constexpr (KIND == 0) v = __int2float_rn((int)r[x]);
                else v = __uint_as_float(r[x]);
                v = __fmul_rn(__fmul_rn(v, sa), sb);
                out[c * 16 + x] = acc_add<ACC>(out[c * 16 + x], v);
              }
            }
          }
        }
        tc_fence_before();
        if constexpr (PAIR == 2) {
          if (leader) mbar_arrive(&acc_empty[buf]);
          else mbar_arrive_remote(buf ? empty_addr1 : empty_addr0);
        } else {
          mbar_arrive(&acc_empty[buf]);
        }
      }
      if (!ok) break;
      // store the finished tile
      if (m < p.m) {
        STO *crow = reinterpret_cast<STO *>(p.c) + ((int64_t)b * p.m + m) * p.ldc;
#pragma unroll
        for (int x = 0; x < NH; ++x) {
          const int cc = n0 + x;
          if (cc < p.n) crow[cc] = to_out<OUTK>(out[x]);
        }
      }
#pragma unroll
      for (int x = 0; x < NH; ++x) out[x] = (ACC)0;
    }
  }

  tc_fence_before();
  if constexpr (PAIR == 2) cluster_sync();   // the peer's TMEM is written by the leader's MMAs
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR == 2) tmem_dealloc_pair(tmem_base, (uint32_t)tcols);
    else tmem_dealloc(tmem_base, (uint32_t)tcols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

int make_map(CUtensorMap *map, const void *base, uint64_t row_bytes, uint64_t rows,
             uint64_t mats, uint32_t box_rows, uint32_t box_mats) {
  auto enc = get_encode();
  if (!enc) return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {row_bytes, rows, mats};
  cuuint64_t strides[2] = {row_bytes, row_bytes * rows};
  cuuint32_t box[3] = {(cuuint32_t)kKBytes, box_rows, box_mats};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return OZ_OK;
}

// Instruction descriptor without the N field (bits 17-22, set per MMA group).
uint32_t make_idesc(int slice_dtype, int mt) {
  uint32_t c_fmt, ab_fmt;
  switch (slice_dtype) {
    case OZ_I8: c_fmt = 2; ab_fmt = 1; break;    // S32 accumulate, signed 8-bit
    case OZ_F16: c_fmt = 1; ab_fmt = 0; break;   // F32 accumulate, F16
    case OZ_BF16: c_fmt = 1; ab_fmt = 1; break;  // F32 accumulate, BF16
    default: c_fmt = 1; ab_fmt = 2; break;       // F32 accumulate, TF32
  }
  uint32_t d = 0;
  d |= c_fmt << 4;
  d |= ab_fmt << 7;
  d |= ab_fmt << 10;
  // bits 15/16 = 0: both operands K-major
  d |= (uint32_t)(mt >> 4) << 24;
  return d;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int KIND, int OUTK, int NT, int PAIR>
int launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const GemmParams &p,
                cudaStream_t st) {
  auto kern = cross_gemm_kernel<KIND, OUTK, NT, PAIR>;
  const int smem = p.stages * stage_bytes(p.s, NT, PAIR, p.pa) + 1024 + kBarrierBytes +
                   scale_stage_bytes(p.s, NT);
  if (int rc = set_smem_once((const void *)kern, smem, "cudaFuncSetAttribute(cross_gemm)"))
    return rc;
  const int units = min(p.num_tiles, sm_count() / PAIR);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(units * PAIR));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, ta, tb, p), "cross_gemm_kernel launch");
}

template <int KIND, int NT, int PAIR>
int launch_out(int out_dtype, const CUtensorMap &ta, const CUtensorMap &tb, const GemmParams &p,
               cudaStream_t st) {
  switch (out_dtype) {
    case OZ_F64: return launch_gemm<KIND, OZ_F64, NT, PAIR>(ta, tb, p, st);
    case OZ_F32: return launch_gemm<KIND, OZ_F32, NT, PAIR>(ta, tb, p, st);
    case OZ_F16: return launch_gemm<KIND, OZ_F16, NT, PAIR>(ta, tb, p, st);
    case OZ_BF16: return launch_gemm<KIND, OZ_BF16, NT, PAIR>(ta, tb, p, st);
    case OZ_I8: return launch_gemm<KIND, OZ_I8, NT, PAIR>(ta, tb, p, st);
  }
  return set_error(OZ_ERR_UNSUPPORTED, "unsupported output dtype %d", out_dtype);
}

template <int NT, int PAIR>
int launch_kind(int kind, int out_dtype, const CUtensorMap &ta, const CUtensorMap &tb,
                const GemmParams &p, cudaStream_t st) {
  if (kind == 0) return launch_out<0, NT, PAIR>(out_dtype, ta, tb, p, st);
  if (kind == 1) return launch_out<1, NT, PAIR>(out_dtype, ta, tb, p, st);
  return launch_out<2, NT, PAIR>(out_dtype, ta, tb, p, st);
}

// Tile shape, raster group and pipeline depth of one launch: the committed
// table (oz_tile_table.h) for the shapes it lists; otherwise NT columns so
// that the s accumulators of one pass fit the 512 TMEM columns, CTA pairs
// (256-row tiles, half the B traffic per CTA) unless M fits one 128-row tile,
// and single-CTA 64-column tiles when a pair grid would leave more than half
// of the SMs idle (they spread a small product over the whole GPU: 0.15 vs
// 0.24 ms for 1024 x 1024 x 8192, s = 4).  OZ_GEMM_TILE="pair,nt" and
// OZ_GEMM_GM override the choice (benchmarking only).
struct TileChoice { int pair, nt, gm, stages; };
TileChoice choose_tile(int kind, int s, int64_t batch, int64_t m, int64_t n, int64_t k) {
  TileChoice t{0, 0, 16, 0};
  bool listed = false;
  for (const TileEntry &e : kTileTable)
    if (e.kind == kind && e.s == s && e.batch == batch && e.m == m && e.n == n && e.k == k &&
        s * e.nt <= 512) {
      t = TileChoice{e.pair, e.nt, e.gm, e.stages};
      listed = true;
      break;
    }
  if (!listed) {
    t.nt = s <= 4 ? 128 : 64;
    t.pair = m > kBM ? 2 : 1;
    const int64_t pair_tiles = batch * ((m + 2 * kBM - 1) / (2 * kBM)) * ((n + t.nt - 1) / t.nt);
    if (t.pair == 2 && pair_tiles * 2 * 2 <= sm_count()) {
      t.pair = 1;
      t.nt = 64;
    }
  }
  if (const char *env = getenv("OZ_GEMM_TILE")) {
    int pr = 0, nt = 0;
    if (sscanf(env, "%d,%d", &pr, &nt) == 2 && (pr == 1 || pr == 2) && (nt == 64 || nt == 128) &&
        s * nt <= 512) {
      t.pair = pr;
      t.nt = nt;
    }
  }
  if (const char *env = getenv("OZ_GEMM_GM")) {
    const int g = atoi(env);
    if (g >= 1 && g <= 64) t.gm = g;
  }
  return t;
}

// Events recorded around the next cross-GEMM launch of this thread
// (oz_profile_next_gemm), then forgotten.
thread_local cudaEvent_t g_prof_begin = nullptr, g_prof_end = nullptr;

}  // namespace
int status_gemm(int *value, bool clear) { return read_status_word(value, clear); }

}  // namespace oz

namespace oz {
namespace {

int cross_gemm_impl(const void *a_slices, const void *b_slices, const float *a_scales,
                    const float *b_scales, int64_t batch, int64_t m, int64_t n, int64_t k,
                    int64_t ld, int32_t num_splits, int slice_dtype, int out_dtype,
                    const int32_t *a_index, const int32_t *b_index, int64_t a_batches,
                    int64_t b_batches, int64_t b_block_cols, void *c, int64_t ldc,
                    uint32_t flags, void *stream, const int32_t *ready = nullptr,
                    int32_t ready_value = 0, int32_t first_block = 0,
                    int32_t block_count = 0) {
  if (num_splits < 1 || num_splits > 8)
    return set_error(OZ_ERR_INVALID, "num_splits must be in [1, 8], got %d", num_splits);
  if (batch < 0 || m < 0 || n < 0 || k < 0)
    return set_error(OZ_ERR_INVALID, "negative size");
  if (slice_dtype != OZ_I8 && slice_dtype != OZ_F16 && slice_dtype != OZ_BF16 &&
      slice_dtype != OZ_F32)
    return set_error(OZ_ERR_UNSUPPORTED, "unsupported slice dtype %d", slice_dtype);
  if (out_dtype != OZ_F64 && out_dtype != OZ_F32 && out_dtype != OZ_F16 && out_dtype != OZ_BF16 &&
      out_dtype != OZ_I8)
    return set_error(OZ_ERR_UNSUPPORTED, "unsupported output dtype %d", out_dtype);
  if (flags & ~OZ_GEMM_SKIP_TAIL) return set_error(OZ_ERR_INVALID, "unknown flags 0x%x", flags);
  if (b_block_cols < 0 || (b_block_cols > 0 && b_block_cols < n && b_block_cols % 128 != 0))
    return set_error(OZ_ERR_INVALID,
                     "B column block width must be 0, >= n or a multiple of 128 (got %lld)",
                     (long long)b_block_cols);
  if (batch == 0 || m == 0 || n == 0) return OZ_OK;
  if (!c || ldc < n) return set_error(OZ_ERR_INVALID, "bad output (ldc=%lld n=%lld)",
                                      (long long)ldc, (long long)n);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int es = dtype_size(slice_dtype);
  const int64_t ld_bytes = ld * es;
  if (k == 0) {
    // empty contraction: C = 0
    if (ldc == n)
      return check_cuda(cudaMemsetAsync(c, 0, (size_t)(batch * m * n * dtype_size(out_dtype)), st),
                        "cudaMemsetAsync");
    return set_error(OZ_ERR_UNSUPPORTED, "k == 0 with a padded output");
  }
  if (!a_slices || !b_slices || !a_scales || !b_scales)
    return set_error(OZ_ERR_INVALID, "null pointer");
  if (ld < k || ld_bytes % kKBytes != 0)
    return set_error(OZ_ERR_INVALID,
                     "slice row pitch must be >= k and a multiple of 128 bytes (ld=%lld)",
                     (long long)ld);
  if (((uintptr_t)a_slices | (uintptr_t)b_slices) % 16 != 0)
    return set_error(OZ_ERR_INVALID, "slice buffers must be 16-byte aligned");
  if (a_batches < 1 || b_batches < 1 || (!a_index && a_batches < batch) ||
      (!b_index && b_batches < batch))
    return set_error(OZ_ERR_INVALID, "bad operand batch counts");
  const int64_t bw = b_block_cols == 0 ? n : b_block_cols;
  const int64_t bblocks = (n + bw - 1) / bw;
  if (ready && (batch != 1 || b_block_cols <= 0 || first_block < 0 || first_block >= bblocks ||
                block_count < 0 || block_count > bblocks))
    return set_error(OZ_ERR_INVALID,
                     "arriving column blocks need batch 1, a block width, a first block in "
                     "[0, %lld) and at most that many blocks (batch=%lld, width=%lld, first=%d, "
                     "count=%d)",
                     (long long)bblocks, (long long)batch, (long long)b_block_cols, first_block,
                     block_count);
  if (m > INT32_MAX || n > INT32_MAX || bw > INT32_MAX || a_batches * num_splits > INT32_MAX ||
      b_batches * bblocks * num_splits > INT32_MAX)
    return set_error(OZ_ERR_INVALID, "size out of range");

  const int kind = slice_dtype == OZ_I8 ? 0 : (slice_dtype == OZ_F32 ? 2 : 1);
  const TileChoice tc = choose_tile(kind, num_splits, batch, m, n, k);
  const int nt = tc.nt, pair = tc.pair;
  // two A slices per pass when both slices' accumulators fit the 512 TMEM
  // columns (s = 2 with 128-column tiles, s <= 4 with 64): the MMA work per
  // fed byte of the pass doubles (C2: 0.63 -> 0.77 of peak; C3 with 64-column
  // single-CTA tiles: 7.26 -> 5.98 ms), at the cost of the double-buffered
  // accumulators when 4 * s * NT > 512.  With an odd num_splits the last pass
  // has one slice; its A box still covers two matrices (the next one lies
  // past the last slice: another batch member's first slice, or outside the
  // tensor, which the copy fills with zeros) and is not multiplied.
  // OZ_GEMM_PA=1 turns it off (benchmarking and tests).
  int pa = (num_splits >= 2 && 2 * num_splits * nt <= 512) ? 2 : 1;
  if (const char *env = getenv("OZ_GEMM_PA"))
    if (atoi(env) == 1) pa = 1;
  CUtensorMap ta, tb;
  // A: one box = the K block of the pass's pa consecutive slices
  if (int rc = make_map(&ta, a_slices, (uint64_t)ld_bytes, (uint64_t)m,
                        (uint64_t)(a_batches * num_splits), kBM, (uint32_t)pa))
    return rc;
  // B: one box = the K block of all num_splits slices, stacked
  // (column blocks: the slices of block c of batch b are matrices (b*blocks + c)*s + j)
  if (int rc = make_map(&tb, b_slices, (uint64_t)ld_bytes, (uint64_t)bw,
                        (uint64_t)(b_batches * bblocks * num_splits), (uint32_t)(nt / pair),
                        (uint32_t)num_splits))
    return rc;

  GemmParams p;
  p.a_scales = a_scales;
  p.b_scales = b_scales;
  p.a_index = a_index;
  p.b_index = b_index;
  p.c = c;
  p.ldc = ldc;
  p.m = (int)m;
  p.n = (int)n;
  p.kblocks = (int)(ld_bytes / kKBytes);
  p.s = num_splits;
  p.skip_tail = (flags & OZ_GEMM_SKIP_TAIL) ? 1 : 0;
  p.batch = (int)batch;
  p.tiles_m = (int)((m + kBM * pair - 1) / (kBM * pair));
  p.tiles_n = (int)((n + nt - 1) / nt);
  p.bw = (int)bw;
  p.bblocks = (int)bblocks;
  p.gm = tc.gm;
  int64_t tiles = (int64_t)p.tiles_m * p.tiles_n * batch;
  if (tiles > INT32_MAX) return set_error(OZ_ERR_INVALID, "too many tiles");
  p.num_tiles = (int)tiles;
  p.idesc = make_idesc(slice_dtype, kBM * pair);
  p.pa = pa;
  p.stages = min(kMaxStages, (kSmemBudget - scale_stage_bytes(num_splits, nt)) /
                                 stage_bytes(num_splits, nt, pair, pa));
  if (tc.stages > 0 && tc.stages < p.stages) p.stages = tc.stages;
  p.ready = ready;
  p.ready_value = ready_value;
  p.first_block = first_block;
  p.tiles_bn = (int)(bw / nt);        // bw is a multiple of 128, nt of 64
  if (ready) {
    tiles = (block_count ? block_count : bblocks) * p.tiles_m * p.tiles_bn;
    if (tiles > INT32_MAX) return set_error(OZ_ERR_INVALID, "too many tiles");
    p.num_tiles = (int)tiles;
  }

  cudaEvent_t ev0 = g_prof_begin, ev1 = g_prof_end;
  g_prof_begin = g_prof_end = nullptr;
  if (ev0)
    if (int rc = check_cuda(cudaEventRecord(ev0, st), "cudaEventRecord(profile begin)")) return rc;
  int rc;
  if (pair == 2)
    rc = nt == 128 ? launch_kind<128, 2>(kind, out_dtype, ta, tb, p, st)
                   : launch_kind<64, 2>(kind, out_dtype, ta, tb, p, st);
  else
    rc = nt == 128 ? launch_kind<128, 1>(kind, out_dtype, ta, tb, p, st)
                   : launch_kind<64, 1>(kind, out_dtype, ta, tb, p, st);
  if (rc == OZ_OK && ev1) rc = check_cuda(cudaEventRecord(ev1, st), "cudaEventRecord(profile end)");
  return rc;
}

}  // namespace
}  // namespace oz

namespace oz {
namespace {
// One thread waits on a shared-memory barrier that nothing arrives on, with
// the same bounded wait the GEMM's roles use, for `bound` SM cycles: the wait
// gives up, records DEV_TIMEOUT_SELFTEST in this unit's status word and the
// kernel returns normally (no trap, the context stays usable).
__global__ void wait_selftest_kernel(long long bound) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  mbar_init(&bar, 1);
  fence_mbar_init();
  abort_flag = 0;
  (void)mbar_wait_bounded(&bar, 0, &abort_flag, DEV_TIMEOUT_SELFTEST, bound);
}
}  // namespace
}  // namespace oz

extern "C" int oz_wait_selftest(int64_t bound_cycles, void *stream) {
  using namespace oz;
  if (bound_cycles <= 0 || bound_cycles > kWaitBoundCycles)
    return set_error(OZ_ERR_INVALID, "bound must be in (0, %lld] cycles", kWaitBoundCycles);
  count_launch();
  wait_selftest_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      (long long)bound_cycles);
  return check_cuda(cudaGetLastError(), "wait_selftest_kernel launch");
}

extern "C" int oz_profile_next_gemm(void *begin_event, void *end_event) {
  oz::g_prof_begin = reinterpret_cast<cudaEvent_t>(begin_event);
  oz::g_prof_end = reinterpret_cast<cudaEvent_t>(end_event);
  return OZ_OK;
}

extern "C" int oz_cross_gemm(const void *a_slices, const void *b_slices, const float *a_scales,
                             const float *b_scales, int64_t batch, int64_t m, int64_t n,
                             int64_t k, int64_t ld, int32_t num_splits, int slice_dtype,
                             int out_dtype, const int32_t *a_index, const int32_t *b_index,
                             int64_t a_batches, int64_t b_batches, void *c, int64_t ldc,
                             uint32_t flags, void *stream) {
  return oz::cross_gemm_impl(a_slices, b_slices, a_scales, b_scales, batch, m, n, k, ld,
                             num_splits, slice_dtype, out_dtype, a_index, b_index, a_batches,
                             b_batches, 0, c, ldc, flags, stream);
}

extern "C" int oz_cross_gemm_blocked(const void *a_slices, const void *b_slices,
                                     const float *a_scales, const float *b_scales, int64_t batch,
                                     int64_t m, int64_t n, int64_t k, int64_t ld,
                                     int32_t num_splits, int slice_dtype, int out_dtype,
                                     const int32_t *a_index, const int32_t *b_index,
                                     int64_t a_batches, int64_t b_batches, int64_t b_block_cols,
                                     void *c, int64_t ldc, uint32_t flags, void *stream) {
  return oz::cross_gemm_impl(a_slices, b_slices, a_scales, b_scales, batch, m, n, k, ld,
                             num_splits, slice_dtype, out_dtype, a_index, b_index, a_batches,
                             b_batches, b_block_cols, c, ldc, flags, stream);
}

extern "C" int oz_cross_gemm_arrivals(const void *a_slices, const void *b_slices,
                                      const float *a_scales, const float *b_scales, int64_t m,
                                      int64_t n, int64_t k, int64_t ld, int32_t num_splits,
                                      int slice_dtype, int out_dtype, int64_t b_block_cols,
                                      const int32_t *ready, int32_t ready_value,
                                      int32_t first_block, int32_t block_count, void *c,
                                      int64_t ldc, uint32_t flags, void *stream) {
  if (!ready) return oz::set_error(OZ_ERR_INVALID, "null arrival flags");
  return oz::cross_gemm_impl(a_slices, b_slices, a_scales, b_scales, 1, m, n, k, ld, num_splits,
                             slice_dtype, out_dtype, nullptr, nullptr, 1, 1, b_block_cols, c, ldc,
                             flags, stream, ready, ready_value, first_block, block_count);
}
