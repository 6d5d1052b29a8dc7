// Shared definitions of the native 3x3 fuse convolution (fuseconv*.cu).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace ddpm {
namespace fuseconv {

constexpr int kSeg = 144;      // staged pixels per source row (128 + 8 on each side)
constexpr int kMaxCin = 256;   // 4C for C <= 64
constexpr int kMaxCout = 64;

// Packed weight images (one per weight version), back to back:
//   forward B chunks   [slab][tap][part][KC/8][Np][8]          (K = input channels)
//   data-grad chunks   [half][slab][tap][part][KD/8][128][8]   (K = output channels)
// `part` = 2 (bf16 hi + residual lo) for FP32 weights, else 1.
struct Layout {
  int Cin, Cout, parts;
  int Np;           // output channels padded to 16 (forward MMA N)
  int KC, nslab;    // forward K slab (input channels) and slab count
  int KD, nslabD;   // data-gradient K slab (output channels) and slab count
  int nhalf;        // data-gradient N blocks of 128 input channels
  size_t fwd_chunk, dg_chunk, fwd_bytes, dg_bytes;
  static Layout make(int cin, int cout, int dt);
};

// Staged source planes of the fuse convolution (input of the forward, output
// gradient of the data gradient): [part][n][G][Hp][Wp][8 channels] in the MMA
// operand type (bf16 hi + residual lo parts for FP32), zero padded: plane row
// i = image row i - 1, plane column j = image column j - 8, channels >= C zero.
// G covers the channels rounded up to 64, so every K slab of either pass is a
// whole number of groups. A unit's 4 rows x 144 columns of one slab are then
// one TMA box per part.
struct PlaneLayout {
  int N, C, H, W, G, Hp, Wp, parts;
  size_t part_bytes;
  size_t bytes() const { return part_bytes * parts; }
  static PlaneLayout make(int n, int c, int h, int w, int dt);
};

}  // namespace fuseconv

size_t fuseconv_pack_bytes(int cin, int cout, int dt);
// gcat_nhwc: write the gradient channel-last [N][H][W][Cin] (Cin % 16 == 0)
int fuseconv_dgrad(const void* gout, const void* packed, void* gcat, int n, int cin, int cout,
                   int h, int w, int dt, cudaStream_t st, int gcat_nhwc = 0);
int fuseconv_dgrad_rowmajor(const void* hi, const void* lo, const void* packed, void* gcat, int n,
                            int cin, int cout, int h, int w, int dt, cudaStream_t st,
                            int gcat_nhwc = 0);

}  // namespace ddpm
