// Out-of-place FP32 transpose, output[c][r] = input[r][c]
// (reference src/transpose.cu:8-47).  Pure data movement: bit-exact.
//
// Aligned shapes (rows and cols multiples of 4, 16-byte aligned pointers) move
// 64x64 tiles with 128-bit loads AND 128-bit stores: a tile is read as float4
// rows into a padded shared tile, and each output float4 is gathered from four
// consecutive tile rows.  The padding (row stride 65 floats) keeps both the
// row writes and the column gathers at most 2-way bank-conflicted.  Other
// shapes use a 32x32 tile with 32-bit accesses (still 128-byte coalesced per
// warp) and bounds checks.
#include <algorithm>

#include "opl_common.cuh"

namespace opl {

constexpr int kT4 = 64;        // tile edge, vector path
constexpr int kT4Threads = 256;

__global__ void __launch_bounds__(kT4Threads)
    transpose_vec4_kernel(const float* __restrict__ input,
                          float* __restrict__ output, int rows, int cols) {
  pdl_begin();
  __shared__ float tile[kT4][kT4 + 1];
  const int tile_col = blockIdx.x * kT4;  // input column origin
  const int c4 = threadIdx.x & 15;        // float4 column inside the tile
  const int r0 = threadIdx.x >> 4;        // 0..15
  const int cols4 = cols >> 2;
  const int rows4 = rows >> 2;
  // Row tiles past grid.y's limit of 65535 continue in grid.z.
  const long long tr = (static_cast<long long>(blockIdx.z) * gridDim.y + blockIdx.y) * kT4;
  if (tr >= rows) return;
  const int tile_row = static_cast<int>(tr);  // input row origin

  // Load: 64 rows x 16 float4, four passes of 16 rows.
  float4 x[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int r = tile_row + r0 + 16 * p;
    const int c = (tile_col >> 2) + c4;
    x[p] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows && c < cols4)
      x[p] = ld_stream(reinterpret_cast<const float4*>(input) +
                       static_cast<std::size_t>(r) * cols4 + c);
  }
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    float* dst = &tile[r0 + 16 * p][4 * c4];
    dst[0] = x[p].x;
    dst[1] = x[p].y;
    dst[2] = x[p].z;
    dst[3] = x[p].w;
  }
  __syncthreads();

  // Store: output row j = input column tile_col + j; output float4 i4 holds
  // input rows tile_row + 4*i4 .. +3.
  const int i4 = threadIdx.x & 15;
  const int j0 = threadIdx.x >> 4;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int j = j0 + 16 * p;
    const int out_row = tile_col + j;
    const int out_c4 = (tile_row >> 2) + i4;
    if (out_row < cols && out_c4 < rows4) {
      const float4 y = make_float4(tile[4 * i4 + 0][j], tile[4 * i4 + 1][j],
                                   tile[4 * i4 + 2][j], tile[4 * i4 + 3][j]);
      st_stream(reinterpret_cast<float4*>(output) +
                    static_cast<std::size_t>(out_row) * rows4 + out_c4,
                y);
    }
  }
}

// Scalar (ragged) path: 32 x 32 tiles, 128 threads of 8 loads each.
// 4097 x 1023: 6.56 us, against 6.65 us with 256 threads of 4 loads,
// 7.2 us with 64 threads of 16, and 7.2 us for 64 x 64 tiles.
constexpr int kT1 = 32;
constexpr int kT1Rows = 4;

__global__ void __launch_bounds__(kT1 * kT1Rows)
    transpose_scalar_kernel(const float* __restrict__ input,
                            float* __restrict__ output, int rows, int cols) {
  pdl_begin();
  __shared__ float tile[kT1][kT1 + 1];
  const int x = blockIdx.x * kT1 + threadIdx.x;
  // Row tiles past grid.y's limit of 65535 continue in grid.z.
  const long long r0l = (static_cast<long long>(blockIdx.z) * gridDim.y + blockIdx.y) * kT1;
  if (r0l >= rows) return;
  const int row0 = static_cast<int>(r0l);
  const int y = row0 + threadIdx.y;
#pragma unroll
  for (int k = 0; k < kT1; k += kT1Rows) {
    if (x < cols && y + k < rows)
      tile[threadIdx.y + k][threadIdx.x] =
          ld_stream(input + static_cast<std::size_t>(y + k) * cols + x);
  }
  __syncthreads();
  const int ox = row0 + threadIdx.x;              // output column (input row)
  const int oy = blockIdx.x * kT1 + threadIdx.y;  // output row (input column)
#pragma unroll
  for (int k = 0; k < kT1; k += kT1Rows) {
    if (ox < rows && oy + k < cols)
      st_stream(output + static_cast<std::size_t>(oy + k) * rows + ox,
                tile[threadIdx.x][threadIdx.y + k]);
  }
}

// Column tiles on x, row tiles on y (at most 65535) and, beyond that, z.
dim3 tile_grid(int rows, int cols, int tile) {
  const int row_tiles = (rows + tile - 1) / tile;
  const int y = std::min(row_tiles, 65535);
  return dim3((cols + tile - 1) / tile, y, (row_tiles + y - 1) / y);
}

}  // namespace opl

extern "C" int opl_transpose_f32(const float* input, float* output, int rows,
                                 int cols, opl_stream_t stream) {
  using namespace opl;
  if (input == nullptr || output == nullptr || rows <= 0 || cols <= 0)
    return cudaErrorInvalidValue;
  if (rows % 4 == 0 && cols % 4 == 0 && aligned16(input) && aligned16(output)) {
    const dim3 grid = tile_grid(rows, cols, kT4);
    return launch_pdl(transpose_vec4_kernel, grid, dim3(kT4Threads), stream, input, output,
                      rows, cols);
  } else {
    const dim3 grid = tile_grid(rows, cols, kT1);
    return launch_pdl(transpose_scalar_kernel, grid, dim3(kT1, kT1Rows), stream, input,
                      output, rows, cols);
  }
  return cudaGetLastError();
}
