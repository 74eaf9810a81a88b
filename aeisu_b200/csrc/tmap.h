// Host-side TMA tensor maps for the chunk-planar activations.
#pragma once

#include <cuda.h>

namespace aeisu {

// A chunk-planar activation t[R][H][nch][W][16 B] seen as a 4-D tensor of 8-byte elements
// {2W, nch, H, R}; the box is one row window {2*win elements (win pixels), box_ch chunks, 1, 1},
// which lands in shared memory as [chunk][pixel][16 B] -- the K-major operand layout of tc.cuh.
// Elements outside the tensor (x < 0, x >= W, y < 0, y >= H) are filled with zeros, which is
// the zero padding of the 3x3 convolutions.  box_ch (default: all nch) chunks per box lets a
// load take one channel group, selected by the chunk coordinate.  win <= 128 (the 256-element
// box limit).
CUtensorMap make_row_window_map(const void* base, int R, int H, int nch, int W, int win, int box_ch = 0);

}  // namespace aeisu
