// Register-cached row kernels: a "group" (one warp, or the whole CTA) owns a
// row, loads it once into registers with coalesced 128-bit (or, for rows that
// are not 16-byte aligned, 32-bit) loads, reduces across the group and writes
// the result, so each row crosses HBM exactly once in each direction.
#pragma once

#include "opl_common.cuh"

namespace opl {

// Shape of a register-cached row launch.  kGroup is 32 (warp per row) or
// kBlock (CTA per row); kItems is the number of float4 (kVec) or float slots
// each thread holds.
struct RowShape {
  int group;
  int block;
  int items;
};

template <bool kVec>
struct RowElems {
  static constexpr int kWidth = kVec ? 4 : 1;
};

// Group-wide reduction.  For kGroup == 32 a warp xor-tree; otherwise a warp
// tree, one slot per warp in `scratch` (kBlock / 32 floats), then every thread
// folds the slots in the same order so all threads hold an identical result.
template <int kGroup, int kBlock, bool kMax>
__device__ __forceinline__ float group_reduce(float v, float* scratch) {
  v = kMax ? warp_max(v) : warp_sum(v);
  if constexpr (kGroup == 32) {
    return v;
  } else {
    static_assert(kGroup == kBlock, "group is a warp or the whole CTA");
    constexpr int kWarps = kBlock / 32;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float r = scratch[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w)
      r = kMax ? fmaxf(r, scratch[w]) : r + scratch[w];
    return r;
  }
}

// Loads the group's row into v[kItems * width]; missing slots get `fill`.
template <int kGroup, int kItems, bool kVec>
__device__ __forceinline__ void load_row(const float* __restrict__ row, int cols,
                                         int t, float fill,
                                         float (&v)[kItems * RowElems<kVec>::kWidth]) {
  if constexpr (kVec) {
    const float4* row4 = reinterpret_cast<const float4*>(row);
    const int vectors = cols >> 2;
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int idx = t + j * kGroup;
      float4 x = make_float4(fill, fill, fill, fill);
      if (idx < vectors) x = ld_stream(row4 + idx);
      v[4 * j + 0] = x.x;
      v[4 * j + 1] = x.y;
      v[4 * j + 2] = x.z;
      v[4 * j + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int col = t + j * kGroup;
      v[j] = col < cols ? ld_stream(row + col) : fill;
    }
  }
}

template <int kGroup, int kItems, bool kVec>
__device__ __forceinline__ void store_row(float* __restrict__ row, int cols, int t,
                                          const float (&v)[kItems * RowElems<kVec>::kWidth]) {
  if constexpr (kVec) {
    float4* row4 = reinterpret_cast<float4*>(row);
    const int vectors = cols >> 2;
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int idx = t + j * kGroup;
      if (idx < vectors)
        st_stream(row4 + idx, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2],
                                          v[4 * j + 3]));
    }
  } else {
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int col = t + j * kGroup;
      if (col < cols) st_stream(row + col, v[j]);
    }
  }
}

// Picks the smallest register-cached shape that holds `count` slots (float4
// slots when vec, float slots otherwise).  Returns false when the row is too
// long for registers and a streaming fallback must be used.
inline bool pick_row_shape(int count, bool vec, RowShape* shape) {
  static const RowShape kVecShapes[] = {
      {32, 128, 1}, {32, 128, 2}, {32, 128, 4}, {32, 128, 8},
      {128, 128, 8}, {256, 256, 8}, {512, 512, 8}, {1024, 1024, 8}};
  static const RowShape kScalarShapes[] = {
      {32, 128, 1}, {32, 128, 2}, {32, 128, 4}, {32, 128, 8}, {32, 128, 16},
      {32, 128, 32}, {128, 128, 32}, {256, 256, 32}, {512, 512, 32},
      {1024, 1024, 32}};
  const RowShape* table = vec ? kVecShapes : kScalarShapes;
  const int entries = vec ? 8 : 10;
  for (int i = 0; i < entries; ++i) {
    if (static_cast<long long>(table[i].group) * table[i].items >= count) {
      *shape = table[i];
      return true;
    }
  }
  return false;
}

// Expands `BODY(kGroup, kBlock, kItems, kVec)` for the shape chosen above.
#define OPL_ROW_DISPATCH(shape, vec, BODY)                                      \
  do {                                                                          \
    if (vec) {                                                                  \
      if (shape.group == 32 && shape.items == 1) BODY(32, 128, 1, true)         \
      else if (shape.group == 32 && shape.items == 2) BODY(32, 128, 2, true)    \
      else if (shape.group == 32 && shape.items == 4) BODY(32, 128, 4, true)    \
      else if (shape.group == 32) BODY(32, 128, 8, true)                        \
      else if (shape.group == 128) BODY(128, 128, 8, true)                      \
      else if (shape.group == 256) BODY(256, 256, 8, true)                      \
      else if (shape.group == 512) BODY(512, 512, 8, true)                      \
      else BODY(1024, 1024, 8, true)                                            \
    } else {                                                                    \
      if (shape.group == 32 && shape.items == 1) BODY(32, 128, 1, false)        \
      else if (shape.group == 32 && shape.items == 2) BODY(32, 128, 2, false)   \
      else if (shape.group == 32 && shape.items == 4) BODY(32, 128, 4, false)   \
      else if (shape.group == 32 && shape.items == 8) BODY(32, 128, 8, false)   \
      else if (shape.group == 32 && shape.items == 16) BODY(32, 128, 16, false) \
      else if (shape.group == 32) BODY(32, 128, 32, false)                      \
      else if (shape.group == 128) BODY(128, 128, 32, false)                    \
      else if (shape.group == 256) BODY(256, 256, 32, false)                    \
      else if (shape.group == 512) BODY(512, 512, 32, false)                    \
      else BODY(1024, 1024, 32, false)                                          \
    }                                                                           \
  } while (0)

}  // namespace opl
