// oz_tile_table.h -- the cross-GEMM's committed tile table.
//
// Replaces the reference's Optuna autotuner (mytuner.py:18-110, applied to the
// GEMM kernel at ozaki_triton.py:292): nothing is searched at run time.  Each
// entry is the fastest tile shape of an event-timed sweep of the kernel on one
// B200 at exactly that shape (the GEMM shapes of the benchmark configurations
// and of their multi-GPU shards; every candidate gives the same bits).  A
// shape that is not listed takes the rule in choose_tile (oz_gemm.cu), which
// reproduces the listed int8 choices.
#pragma once

#include <stdint.h>

namespace oz {

struct TileEntry {
  int kind;                  // slice kind: 0 int8, 1 fp16 / bf16, 2 tf32 (fp32 slices)
  int s;                     // num_splits
  int64_t batch, m, n, k;    // the product's shape (n: columns of one launch)
  int pair;                  // 2: CTA pair, 256-row tiles; 1: one CTA, 128-row tiles
  int nt;                    // tile columns (s * nt <= 512 TMEM columns)
  int gm;                    // row tiles per raster group
  int stages;                // pipeline stages (0: as many as shared memory holds)
};

// kind, s, batch, m, n, k, pair, nt, gm, stages          sweep (ms): chosen / next best
constexpr TileEntry kTileTable[] = {
    // C1: FP32 -> FP16 s=2, 256^3                        0.029 / 0.036 (1,128)
    {1, 2, 1, 256, 256, 256, 2, 64, 16, 0},
    // C3: FP64 -> INT8 8192^3 (s = 4 headline; 6, 8 with the fp64 residual)
    {0, 4, 1, 8192, 8192, 8192, 2, 128, 16, 0},        // 7.07 / 8.30 (1,128)
    {0, 6, 1, 8192, 8192, 8192, 2, 64, 16, 0},         // 18.95 / 19.20 (1,64)
    {0, 8, 1, 8192, 8192, 8192, 2, 64, 16, 0},         // 28.87 / 31.99 (1,64)
    // C4: FP64 -> FP16 s=3, 128 x (2048 x 2048 x 4096) from 16 x 8 operands
    {1, 3, 128, 2048, 2048, 4096, 1, 128, 16, 0},      // 42.15 / 44.45 (2,128)
    // C4 on 8 GPUs: 16 output batches per rank
    {1, 3, 16, 2048, 2048, 4096, 1, 128, 16, 0},       // 4.96 / 5.38 (2,128)
    // C5: FP64 -> INT8 16384^3
    {0, 4, 1, 16384, 16384, 16384, 2, 128, 16, 0},     // 61.5 / 63.0 (1,128)
    {0, 6, 1, 16384, 16384, 16384, 2, 64, 16, 0},      // 163.4 / 172.5 (1,64)
    {0, 8, 1, 16384, 16384, 16384, 2, 64, 16, 0},      // 252.9 / 258.5 (1,64)
    // shards of C3 / C5 on 2-8 GPUs (rows of A x all of N, or x one column block)
    {0, 4, 1, 2048, 8192, 8192, 2, 128, 16, 0},        // 1.578 / 1.861 (1,128)
    // the 8-GPU p2p blocks (1024 rows x 1024 columns): one block alone 0.163 ms
    // vs 0.170 (2,64) with one A slice per pass (these 64-column tiles now
    // take two per pass).  A 1-GPU emulation of a rank's eight block GEMMs with
    // all blocks present favoured (2,128) on one stream per block (0.835 vs
    // 0.926 ms), but on 8 GPUs, with blocks arriving one by one, that setting
    // gave 1043 TFLOPS against 1107 for this entry with 2 GEMM streams
    {0, 4, 1, 1024, 1024, 8192, 1, 64, 16, 0},
    // one rank's 1024 rows x all 8192 columns (eight 1024-column blocks) in one
    // launch, every block present:      0.778 / 0.811 (2,64); 0.851 (2,128)
    {0, 4, 1, 1024, 8192, 8192, 1, 64, 16, 0},
    {0, 4, 1, 2048, 16384, 16384, 2, 128, 16, 0},      // 6.73 / 8.32 (1,128)
};

}  // namespace oz
