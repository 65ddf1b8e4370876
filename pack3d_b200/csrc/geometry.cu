// Native builders of the geometry tables (reference geometry.py:54-101, 190-266): the
// neighbour table of a complete voxel stencil and its transport under a repack, each with
// the sorted-row table that is the reverse adjacency of a symmetric graph.  Host code only,
// multithreaded over rows; bit-identical to pack3d_b200.geometry's tensor formulation:
//
//   neighbors[i][k] = packed row of raster(coords(order[i]) + offset_k), -1 outside the grid,
//                     offsets in itertools.product order (z-major, -r .. r per axis);
//   sorted[i]       = the row's valid entries in ascending order, -1 padding last
//                     (where(nb >= 0, nb, N).sort() with N -> -1);
//   max_valid       = the largest count of valid entries in a row (the reverse table's width).
#include <algorithm>
#include <thread>
#include <vector>

#include "common.cuh"

namespace p3d {
namespace {

// Run body(lo, hi) -> int over row ranges on `threads` threads (0: all hardware threads);
// returns the maximum of the results.
template <typename F>
int parallel_rows_max(int64_t n, int threads, F &&body) {
  if (threads < 1) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  const int64_t per = std::max<int64_t>(4096, (n + threads - 1) / threads);
  const int64_t parts = (n + per - 1) / per;
  std::vector<int> result((size_t)std::max<int64_t>(parts, 1), 0);
  std::vector<std::thread> pool;
  for (int64_t w = 0; w < parts; ++w) {
    const int64_t lo = w * per, hi = std::min(n, lo + per);
    pool.emplace_back([&body, &result, w, lo, hi] { result[(size_t)w] = body(lo, hi); });
  }
  for (auto &t : pool) t.join();
  return *std::max_element(result.begin(), result.end());
}

// Sorted copy of one row (valid entries ascending, -1 last); returns the valid count.
int sort_row(const int32_t *row, int width, int32_t *out) {
  int c = 0;
  for (int k = 0; k < width; ++k)
    if (row[k] >= 0) out[c++] = row[k];
  std::sort(out, out + c);
  for (int k = c; k < width; ++k) out[k] = -1;
  return c;
}

// inverse[order[i]] = i; false unless order is a permutation of [0, n)
bool invert(const int64_t *order, int64_t n, std::vector<int32_t> &inverse) {
  inverse.assign((size_t)n, -1);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t r = order[i];
    if (r < 0 || r >= n || inverse[(size_t)r] >= 0) return false;
    inverse[(size_t)r] = (int32_t)i;
  }
  return true;
}

}  // namespace
}  // namespace p3d

using namespace p3d;

extern "C" int p3d_stencil_neighbors(int Z, int Y, int X, int rz, int ry, int rx, const int64_t *order, int64_t n,
                                     int32_t *neighbors, int32_t *sorted, int32_t *max_valid, int threads) {
  P3D_CHECK_ARG(Z >= 1 && Y >= 1 && X >= 1 && (int64_t)Z * Y * X == n, "p3d_stencil_neighbors: bad grid");
  P3D_CHECK_ARG(rz >= 0 && ry >= 0 && rx >= 0 && (2 * rz + 1) * (2 * ry + 1) * (2 * rx + 1) <= 128,
                "p3d_stencil_neighbors: bad radius");
  P3D_CHECK_ARG(order && neighbors && sorted && max_valid, "p3d_stencil_neighbors: null pointer");
  P3D_CHECK_ARG(n < (int64_t(1) << 31), "p3d_stencil_neighbors: more than 2^31 tokens");
  const int width = (2 * rz + 1) * (2 * ry + 1) * (2 * rx + 1);
  std::vector<int32_t> inverse;
  P3D_CHECK_ARG(invert(order, n, inverse), "p3d_stencil_neighbors: order is not a permutation");
  const int64_t plane = (int64_t)Y * X;
  *max_valid = parallel_rows_max(n, threads, [&](int64_t lo, int64_t hi) {
    int best = 0;
    for (int64_t i = lo; i < hi; ++i) {
      const int64_t r = order[i];
      const int z = (int)(r / plane), y = (int)((r / X) % Y), x = (int)(r % X);
      int32_t *row = neighbors + i * width;
      int k = 0;
      for (int dz = -rz; dz <= rz; ++dz)
        for (int dy = -ry; dy <= ry; ++dy)
          for (int dx = -rx; dx <= rx; ++dx, ++k) {
            const int tz = z + dz, ty = y + dy, tx = x + dx;
            const bool in = tz >= 0 && tz < Z && ty >= 0 && ty < Y && tx >= 0 && tx < X;
            row[k] = in ? inverse[(size_t)(((int64_t)tz * Y + ty) * X + tx)] : -1;
          }
      best = std::max(best, sort_row(row, width, sorted + i * width));
    }
    return best;
  });
  return P3D_OK;
}

extern "C" int p3d_repack_neighbors(int64_t n, int width, const int32_t *nb_old, const int64_t *perm,
                                    int32_t *nb_new, int32_t *sorted, int32_t *max_valid, int threads) {
  P3D_CHECK_ARG(n >= 1 && n < (int64_t(1) << 31) && width >= 1 && width <= 128, "p3d_repack_neighbors: bad shape");
  P3D_CHECK_ARG(nb_old && perm && nb_new && sorted && max_valid, "p3d_repack_neighbors: null pointer");
  std::vector<int32_t> inverse;
  P3D_CHECK_ARG(invert(perm, n, inverse), "p3d_repack_neighbors: not a permutation");
  for (int64_t i = 0; i < n * width; ++i)
    P3D_CHECK_ARG(nb_old[i] >= -1 && nb_old[i] < n, "p3d_repack_neighbors: out-of-range neighbour");
  *max_valid = parallel_rows_max(n, threads, [&](int64_t lo, int64_t hi) {
    int best = 0;
    for (int64_t i = lo; i < hi; ++i) {
      const int32_t *src = nb_old + perm[i] * width;
      int32_t *row = nb_new + i * width;
      for (int k = 0; k < width; ++k) row[k] = src[k] >= 0 ? inverse[(size_t)src[k]] : -1;
      best = std::max(best, sort_row(row, width, sorted + i * width));
    }
    return best;
  });
  return P3D_OK;
}
