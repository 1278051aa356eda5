// DB post-processing front end on the device: 8-connected components of the
// binarized probability map with per-component box statistics, so the host
// reads a few KB of candidates instead of the full FP32 map.
//
// Reference: postprocess_db_map_opencv (native/src/detection/
// db_postprocess.cpp:183-252) binarizes the map (cv::compare, 189-190), then
// cv::findContours(RETR_LIST) walks the 8-connected foreground components'
// boundaries on the host and scores each candidate box on the FP32 map
// (box_score_fast). Here the components come out labelled with
// (left, top, width, height, area) per component, numbered exactly as
// OpenCV's connectedComponentsWithStats(connectivity 8) numbers them (the
// tests' oracle): in order of each component's first pixel in 2x2-block
// raster order, key(y, x) = ((y/2) * ceil(W/2) + x/2) * 4 + (y%2) * 2 + x%2,
// the order in which OpenCV's block-based labelling hands out provisional
// labels. Each component also gets the sum of its pixels' probabilities in
// 32.32 fixed point (integer atomics: deterministic).
//
// Labelling is union-find over keys (a root is always the smallest key of
// its tree: a link only ever points a larger root at a smaller one, by
// atomicMin), in passes over the page: (1) each 32 x 32 tile (whole 2x2
// blocks) is labelled in shared memory, its local index order being the
// key order, and every pixel's global entry points at its tile-local root;
// (2) pixels with a neighbour in another tile unite the trees in global
// memory; (3) path compression; (4) numbering of the roots by a per-page
// exclusive scan in key order; (5) one labelling/statistics pass. A plain
// pixel-level union-find measured 1.9 ms on 8 DB-like pages of 960^2
// (row-long chains); the tile pass keeps global trees shallow.
#include "kernels.h"
#include <climits>

namespace pb2 {
namespace {

constexpr int kCclThreads = 256;
constexpr int kScanBlock = 1024; // keys per scan block

struct Geo {
  int H, W, Wb;     // image, blocks per block row
  long long kp;     // keys per page: 4 * ceil(H/2) * Wb
  long long hw;     // pixels per page
};

__device__ __forceinline__ long long key_of(const Geo &g, int y, int x) {
  return ((static_cast<long long>(y >> 1) * g.Wb + (x >> 1)) << 2) + ((y & 1) << 1) + (x & 1);
}

__device__ __forceinline__ int find_root(const int *__restrict__ lab, int x) {
  int p = lab[x];
  while (p != x) {
    x = p;
    p = lab[x];
  }
  return x;
}

// Links the trees of a and b; the larger root is pointed at the smaller.
__device__ void unite(int *lab, int a, int b) {
  while (true) {
    a = find_root(lab, a);
    b = find_root(lab, b);
    if (a == b)
      return;
    if (a > b) {
      const int t = a;
      a = b;
      b = t;
    }
    // b is a root larger than a: point it at a unless another thread has
    // linked it meanwhile; then retry from the parent it got (the link that
    // atomicMin may have replaced is restored by that retry).
    const int old = atomicMin(&lab[b], a);
    if (old == b)
      return;
    b = old;
  }
}

constexpr int kTile = 32; // tile edge in pixels (16 x 16 blocks of 2 x 2)

// Unions only with the neighbours that are not already joined through
// another one (8-connectivity): `up` covers up-left and up-right (each is a
// horizontal neighbour of `up`, joined by its own pixel's pass); `left`
// covers up-left (left's own up).
template <class Fg, class Unite>
__device__ __forceinline__ void unite_previous(bool has_left, bool has_up, bool has_right, Fg fg, Unite un) {
  const bool up = has_up && fg(-1, 0);
  if (up) {
    un(-1, 0);
    return;
  }
  const bool left = has_left && fg(0, -1);
  if (left)
    un(0, -1);
  else if (has_left && has_up && fg(-1, -1))
    un(-1, -1);
  if (has_right && has_up && fg(-1, 1))
    un(-1, 1);
}

// (1) Tile pass: 1024 threads = 32 x 32 pixels of one tile; every key of the
// tile (padding keys of odd sizes included) gets its entry: -1 for
// background, else the global key of the pixel's tile-local root.
__global__ void __launch_bounds__(kTile * kTile)
    ccl_tile_kernel(const uint8_t *__restrict__ bitmap, int *__restrict__ lab, Geo g, int tiles_x, int tiles_y) {
  __shared__ int sl[kTile * kTile];
  const int tx = threadIdx.x & (kTile - 1), ty = threadIdx.x / kTile;
  const int tile = blockIdx.x;
  const int page = tile / (tiles_x * tiles_y), tr = tile % (tiles_x * tiles_y);
  const int y0 = (tr / tiles_x) * kTile, x0 = (tr % tiles_x) * kTile;
  const int y = y0 + ty, x = x0 + tx;
  // local index in key order: 2x2 blocks raster over the tile, then the
  // pixel's place in its block
  const int L = (((ty >> 1) * (kTile / 2) + (tx >> 1)) << 2) + ((ty & 1) << 1) + (tx & 1);
  const uint8_t *bm = bitmap + static_cast<long long>(page) * g.hw;
  auto fg_at = [&](int yy, int xx) { return yy < g.H && xx < g.W && bm[static_cast<long long>(yy) * g.W + xx] != 0; };
  const bool me = fg_at(y, x);
  sl[L] = me ? L : -1;
  __syncthreads();
  if (me) {
    auto lidx = [&](int dy, int dx) {
      const int a = ty + dy, b = tx + dx;
      return (((a >> 1) * (kTile / 2) + (b >> 1)) << 2) + ((a & 1) << 1) + (b & 1);
    };
    unite_previous(tx > 0, ty > 0, tx + 1 < kTile, [&](int dy, int dx) { return fg_at(y + dy, x + dx); },
                   [&](int dy, int dx) { unite(sl, L, lidx(dy, dx)); });
  }
  __syncthreads();
  // Keys of the tile's padding rows/columns beyond the image are inside the
  // page's key space only where the image ends mid-block; they stay -1.
  if (y < ((g.H + 1) & ~1) && x < ((g.W + 1) & ~1)) {
    int v = -1;
    if (me) {
      const int r = find_root(sl, L);
      const int rq = r & 3, rb = r >> 2;
      const int ry = y0 + (rb / (kTile / 2)) * 2 + (rq >> 1), rx = x0 + (rb % (kTile / 2)) * 2 + (rq & 1);
      v = static_cast<int>(static_cast<long long>(page) * g.kp + key_of(g, ry, rx));
    }
    lab[static_cast<long long>(page) * g.kp + key_of(g, y, x)] = v;
  }
}

// (2) Unites across tile borders. A pixel's previous neighbours (left,
// up-left, up, up-right) leave its tile only on the tile's top row, left
// column or right column; one thread per such pixel (96 per tile, corners
// twice, which is harmless) joins the trees in global memory.
__global__ void __launch_bounds__(3 * kTile)
    ccl_border_kernel(const uint8_t *__restrict__ bitmap, int *lab, Geo g, int tiles_x, int tiles_y) {
  const int tile = blockIdx.x;
  const int page = tile / (tiles_x * tiles_y), tr = tile % (tiles_x * tiles_y);
  const int y0 = (tr / tiles_x) * kTile, x0 = (tr % tiles_x) * kTile;
  const int side = threadIdx.x / kTile, t = threadIdx.x % kTile;
  const int y = side == 0 ? y0 : y0 + t;
  const int x = side == 0 ? x0 + t : (side == 1 ? x0 : x0 + kTile - 1);
  if (y >= g.H || x >= g.W)
    return;
  const uint8_t *bm = bitmap + static_cast<long long>(page) * g.hw;
  if (!bm[static_cast<long long>(y) * g.W + x])
    return;
  const long long base = static_cast<long long>(page) * g.kp;
  const int me = static_cast<int>(base + key_of(g, y, x));
  auto link = [&](int yy, int xx) {
    const bool other = yy < y0 || xx < x0 || xx >= x0 + kTile;
    if (other && bm[static_cast<long long>(yy) * g.W + xx])
      unite(lab, me, static_cast<int>(base + key_of(g, yy, xx)));
  };
  if (x > 0)
    link(y, x - 1);
  if (y > 0) {
    link(y - 1, x);
    if (x > 0)
      link(y - 1, x - 1);
    if (x + 1 < g.W)
      link(y - 1, x + 1);
  }
}

// Scan block b covers keys [bb * 1024, (bb + 1) * 1024) of page b / bpp
// (bb = b % bpp), so no block holds two pages' keys.
__device__ __forceinline__ long long scan_key(const Geo &g, int bpp, bool &inside) {
  const int page = blockIdx.x / bpp, bb = blockIdx.x - page * bpp;
  const long long local = static_cast<long long>(bb) * kScanBlock + threadIdx.x;
  inside = local < g.kp;
  return page * g.kp + local;
}

// Path compression; also counts the roots of each scan block.
__global__ void __launch_bounds__(kScanBlock)
    ccl_compress_kernel(int *lab, Geo g, int bpp, int *__restrict__ block_roots) {
  bool inside;
  const long long k = scan_key(g, bpp, inside);
  int root = 0;
  if (inside && lab[k] >= 0) {
    const int r = find_root(lab, static_cast<int>(k));
    lab[k] = r;
    root = r == static_cast<int>(k);
  }
  const int cnt = __syncthreads_count(root);
  if (threadIdx.x == 0)
    block_roots[blockIdx.x] = cnt;
}

// Exclusive scan of the per-block root counts, restarting at every page
// (page p owns scan blocks [p * bpp, (p + 1) * bpp)): one block per page,
// 1024 counts per round (warp scans, then a scan of the warp totals).
__global__ void __launch_bounds__(1024)
    ccl_scan_pages_kernel(const int *__restrict__ block_roots, int *__restrict__ block_base, int bpp,
                          int *__restrict__ counts) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  const int p = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0)
    carry = 0;
  __syncthreads();
  for (int b0 = 0; b0 < bpp; b0 += 1024) {
    const int b = b0 + threadIdx.x;
    const int v = b < bpp ? block_roots[p * bpp + b] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o)
        incl += t;
    }
    if (lane == 31)
      warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int w = warp_tot[lane];
      int wi = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o)
          wi += t;
      }
      warp_tot[lane] = wi - w; // exclusive over warps
    }
    __syncthreads();
    const int base = carry;
    if (b < bpp)
      block_base[p * bpp + b] = base + warp_tot[warp] + incl - v;
    __syncthreads();
    if (threadIdx.x == 1023)
      carry = base + warp_tot[warp] + incl;
    __syncthreads();
  }
  if (threadIdx.x == 0)
    counts[p] = carry;
}

// Component number of every root: its page's block base plus its rank in
// the block (roots in increasing key order).
__global__ void __launch_bounds__(kScanBlock)
    ccl_number_kernel(const int *__restrict__ lab, Geo g, int bpp, const int *__restrict__ block_base,
                      int *__restrict__ rankmap) {
  __shared__ int warp_sums[kScanBlock / 32];
  bool inside;
  const long long k = scan_key(g, bpp, inside);
  const bool root = inside && lab[k] == static_cast<int>(k);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned ballot = __ballot_sync(0xffffffffu, root);
  const int in_warp = __popc(ballot & ((1u << lane) - 1u));
  if (lane == 0)
    warp_sums[warp] = __popc(ballot);
  __syncthreads();
  if (warp == 0) {
    const int own = warp_sums[lane];
    int v = own;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o)
        v += t;
    }
    warp_sums[lane] = v - own; // exclusive
  }
  __syncthreads();
  if (root)
    rankmap[k] = block_base[blockIdx.x] + warp_sums[warp] + in_warp;
}

__global__ void __launch_bounds__(kCclThreads)
    ccl_stats_init_kernel(int *__restrict__ bbox, int *__restrict__ area, unsigned long long *__restrict__ probq,
                          long long slots) {
  const long long i = static_cast<long long>(blockIdx.x) * kCclThreads + threadIdx.x;
  if (i >= slots)
    return;
  bbox[4 * i + 0] = INT_MAX; // min x
  bbox[4 * i + 1] = INT_MAX; // min y
  bbox[4 * i + 2] = -1;      // max x
  bbox[4 * i + 3] = -1;      // max y
  area[i] = 0;
  probq[i] = 0ull;
}

// Final labels (1..N per page, 0 background) and the per-component
// accumulations: bbox extremes, area, fixed-point probability sum. Lanes of
// a warp holding the same component (a run of pixels of one row, usually)
// are combined first (match + warp reductions), so a large component costs
// one set of atomics per warp instead of one per pixel: per-pixel atomics on
// the few hot addresses of big text blobs measured 1.0 ms on 8 pages.
__global__ void __launch_bounds__(kCclThreads)
    ccl_label_stats_kernel(const int *__restrict__ lab, const int *__restrict__ rankmap,
                           const float *__restrict__ prob, Geo g, long long n, int max_comp,
                           int *__restrict__ labels, int *__restrict__ bbox, int *__restrict__ area,
                           unsigned long long *__restrict__ probq) {
  const long long i = static_cast<long long>(blockIdx.x) * kCclThreads + threadIdx.x;
  long long slot = -1;
  int x = 0, y = 0;
  uint32_t fixed = 0, fixed_hi = 0;
  if (i < n) {
    const long long page = i / g.hw, pl = i - page * g.hw;
    y = static_cast<int>(pl / g.W);
    x = static_cast<int>(pl - static_cast<long long>(y) * g.W);
    const int r = lab[page * g.kp + key_of(g, y, x)];
    if (r < 0) {
      labels[i] = 0;
    } else {
      const int id = rankmap[r]; // 0-based component number in its page
      labels[i] = id + 1;
      if (id < max_comp) {
        slot = page * max_comp + id;
        if (prob) {
          const float pv = fminf(fmaxf(prob[i], 0.0f), 1.0f);
          // 32.32 fixed point: floor(p * 2^32), exact in double; <= 2^32.
          const unsigned long long q = static_cast<unsigned long long>(static_cast<double>(pv) * 4294967296.0);
          fixed = static_cast<uint32_t>(q & 0xFFFFu);
          fixed_hi = static_cast<uint32_t>(q >> 16);
        }
      }
    }
  }
  // Group the warp's lanes by slot (-1: nothing to add).
  const unsigned grp = __match_any_sync(0xffffffffu, slot);
  const int xmin = static_cast<int>(__reduce_min_sync(grp, static_cast<unsigned>(x)));
  const int ymin = static_cast<int>(__reduce_min_sync(grp, static_cast<unsigned>(y)));
  const int xmax = static_cast<int>(__reduce_max_sync(grp, static_cast<unsigned>(x)));
  const int ymax = static_cast<int>(__reduce_max_sync(grp, static_cast<unsigned>(y)));
  // each part <= 2^16, so 32 lanes' sums fit in 32 bits
  const unsigned lo = __reduce_add_sync(grp, fixed);
  const unsigned hi = __reduce_add_sync(grp, fixed_hi);
  const int lane = threadIdx.x & 31;
  if (slot >= 0 && lane == __ffs(grp) - 1) {
    atomicMin(&bbox[4 * slot + 0], xmin);
    atomicMin(&bbox[4 * slot + 1], ymin);
    atomicMax(&bbox[4 * slot + 2], xmax);
    atomicMax(&bbox[4 * slot + 3], ymax);
    atomicAdd(&area[slot], __popc(grp));
    if (prob)
      atomicAdd(&probq[slot], (static_cast<unsigned long long>(hi) << 16) + lo);
  }
}

// (min x, min y, max x, max y) -> OpenCV's (left, top, width, height, area).
__global__ void __launch_bounds__(kCclThreads)
    ccl_stats_finish_kernel(const int *__restrict__ bbox, const int *__restrict__ area, int *__restrict__ stats,
                            const int *__restrict__ counts, int max_comp, long long slots) {
  const long long i = static_cast<long long>(blockIdx.x) * kCclThreads + threadIdx.x;
  if (i >= slots)
    return;
  const int page = static_cast<int>(i / max_comp), id = static_cast<int>(i % max_comp);
  int *o = stats + 5 * i;
  if (id >= counts[page]) {
    o[0] = o[1] = o[2] = o[3] = o[4] = 0;
    return;
  }
  o[0] = bbox[4 * i + 0];
  o[1] = bbox[4 * i + 1];
  o[2] = bbox[4 * i + 2] - bbox[4 * i + 0] + 1;
  o[3] = bbox[4 * i + 3] - bbox[4 * i + 1] + 1;
  o[4] = area[i];
}

long long blocks(long long n, int t) { return (n + t - 1) / t; }
size_t al256(long long b) { return static_cast<size_t>((b + 255) / 256 * 256); }

Geo geometry(int H, int W) {
  Geo g;
  g.H = H;
  g.W = W;
  g.Wb = (W + 1) / 2;
  g.kp = 4LL * ((H + 1) / 2) * g.Wb;
  g.hw = static_cast<long long>(H) * W;
  return g;
}

} // namespace

size_t db_components_workspace(int pages, int H, int W, int max_comp) {
  const Geo g = geometry(H, W);
  const long long bpp = (g.kp + kScanBlock - 1) / kScanBlock;
  const long long slots = static_cast<long long>(pages) * max_comp;
  // key labels + rankmap (int per key), block roots + block bases, bbox (4
  // ints per slot), area (int per slot); each 256-byte aligned.
  return 2 * al256(4 * pages * g.kp) + 2 * al256(4 * pages * bpp) + al256(16 * slots) + al256(4 * slots);
}

cudaError_t db_components(const uint8_t *bitmap, const float *prob, int pages, int H, int W, int max_comp,
                          int *labels, int *counts, int *stats, unsigned long long *probq, void *workspace,
                          cudaStream_t s) {
  if (pages <= 0 || H <= 0 || W <= 0)
    return cudaSuccess;
  const Geo g = geometry(H, W);
  const long long n = g.hw * pages, nk = g.kp * pages;
  if (nk >= (1LL << 31) || max_comp <= 0 || !bitmap || !labels || !counts || !stats || !probq || !workspace)
    return cudaErrorInvalidValue;
  const long long bpp = (g.kp + kScanBlock - 1) / kScanBlock;
  const long long slots = static_cast<long long>(pages) * max_comp;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  int *klab = reinterpret_cast<int *>(ws);
  ws += al256(4 * nk);
  int *rankmap = reinterpret_cast<int *>(ws);
  ws += al256(4 * nk);
  int *block_roots = reinterpret_cast<int *>(ws);
  ws += al256(4 * pages * bpp);
  int *block_base = reinterpret_cast<int *>(ws);
  ws += al256(4 * pages * bpp);
  int *bbox = reinterpret_cast<int *>(ws);
  ws += al256(16 * slots);
  int *area = reinterpret_cast<int *>(ws);
  const unsigned scan_blocks = static_cast<unsigned>(pages * bpp);
  const int tiles_x = (W + kTile - 1) / kTile, tiles_y = (H + kTile - 1) / kTile;
  ccl_tile_kernel<<<static_cast<unsigned>(static_cast<long long>(pages) * tiles_x * tiles_y), kTile * kTile, 0, s>>>(
      bitmap, klab, g, tiles_x, tiles_y);
  ccl_border_kernel<<<static_cast<unsigned>(static_cast<long long>(pages) * tiles_x * tiles_y), 3 * kTile, 0, s>>>(
      bitmap, klab, g, tiles_x, tiles_y);
  ccl_stats_init_kernel<<<blocks(slots, kCclThreads), kCclThreads, 0, s>>>(bbox, area, probq, slots);
  ccl_compress_kernel<<<scan_blocks, kScanBlock, 0, s>>>(klab, g, static_cast<int>(bpp), block_roots);
  ccl_scan_pages_kernel<<<pages, 1024, 0, s>>>(block_roots, block_base, static_cast<int>(bpp), counts);
  ccl_number_kernel<<<scan_blocks, kScanBlock, 0, s>>>(klab, g, static_cast<int>(bpp), block_base, rankmap);
  ccl_label_stats_kernel<<<blocks(n, kCclThreads), kCclThreads, 0, s>>>(klab, rankmap, prob, g, n, max_comp, labels,
                                                                         bbox, area, probq);
  ccl_stats_finish_kernel<<<blocks(slots, kCclThreads), kCclThreads, 0, s>>>(bbox, area, stats, counts, max_comp,
                                                                             slots);
  return cudaGetLastError();
}

} // namespace pb2
