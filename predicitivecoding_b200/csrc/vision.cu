// Annotation rasteriser on a device RGB buffer (headless): box outlines and line segments.
//
// Reference counterpart: PredictiveCoding.Vision/Annotate.cs:11-117 (CPU: clamped box outlines of
// thickness t drawn as horizontal/vertical runs, all-octant integer Bresenham segments, later
// primitives painting over earlier ones).  Here every primitive rasterises in parallel (boxes:
// one block per box, threads over outline pixels; segments: one thread per segment walking the
// same Bresenham recurrence) and records its index with atomicMax in an owner map; a resolve
// pass paints each owned pixel with its highest-index (= latest) primitive's colour, so the result
// is the CPU drawing order's, pixel for pixel.
#include <cuda_runtime.h>
#include <cstdint>

namespace {

__device__ __forceinline__ void own(int* owner, int W, int H, int x, int y, int prim) {
  if ((unsigned)x < (unsigned)W && (unsigned)y < (unsigned)H) atomicMax(owner + y * W + x, prim);
}

// boxes: [n, 4] int (x1, y1, x2, y2) already clamped to the image; thickness t
__global__ void box_kernel(const int* __restrict__ boxes, int n, int t, int* __restrict__ owner, int W, int H) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const int x1 = boxes[4 * i], y1 = boxes[4 * i + 1], x2 = boxes[4 * i + 2], y2 = boxes[4 * i + 3];
  const int wlen = max(0, x2 - x1 + 1), hlen = max(0, y2 - y1 + 1);
  const int per_k = 2 * wlen + 2 * hlen;
  for (int j = threadIdx.x; j < per_k * t; j += blockDim.x) {
    const int k = j / per_k, r = j % per_k;
    if (r < wlen) own(owner, W, H, x1 + r, y1 + k, i);
    else if (r < 2 * wlen) own(owner, W, H, x1 + r - wlen, y2 - k, i);
    else if (r < 2 * wlen + hlen) own(owner, W, H, x1 + k, y1 + r - 2 * wlen, i);
    else own(owner, W, H, x2 - k, y1 + r - 2 * wlen - hlen, i);
  }
}

// segments: [m, 4] int (x0, y0, x1, y1); primitive index = base + s
__global__ void segment_kernel(const int* __restrict__ seg, int m, int base, int* __restrict__ owner, int W, int H,
                               int max_steps) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= m) return;
  int x0 = seg[4 * s], y0 = seg[4 * s + 1];
  const int x1 = seg[4 * s + 2], y1 = seg[4 * s + 3];
  const int dx = abs(x1 - x0), sx = x0 < x1 ? 1 : -1;
  const int dy = -abs(y1 - y0), sy = y0 < y1 ? 1 : -1;
  int err = dx + dy;
  for (int step = 0; step <= max_steps; ++step) {   // bounded: a segment has at most dx - dy + 1 pixels
    own(owner, W, H, x0, y0, base + s);
    if (x0 == x1 && y0 == y1) break;
    const int e2 = 2 * err;
    if (e2 >= dy) { err += dy; x0 += sx; }
    if (e2 <= dx) { err += dx; y0 += sy; }
  }
}

__global__ void resolve_kernel(const int* __restrict__ owner, const uint8_t* __restrict__ colors,
                               uint8_t* __restrict__ img, int npix) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= npix) return;
  const int o = owner[p];
  if (o < 0) return;
  img[3 * p] = colors[3 * o];
  img[3 * p + 1] = colors[3 * o + 1];
  img[3 * p + 2] = colors[3 * o + 2];
}

}  // namespace

// img [H, W, 3] uint8 (device); owner [H*W] int32 scratch (set to -1 here); colors [(n+m), 3] uint8.
int pcb_annotate(uint8_t* img, int W, int H, const int* boxes, int n, int thickness, const int* segs, int m,
                 const uint8_t* colors, int* owner, cudaStream_t s) {
  if (W <= 0 || H <= 0 || thickness < 1) return -2;
  cudaMemsetAsync(owner, 0xFF, sizeof(int) * (size_t)W * H, s);
  if (n > 0) box_kernel<<<n, 256, 0, s>>>(boxes, n, thickness, owner, W, H);
  if (m > 0) segment_kernel<<<(m + 127) / 128, 128, 0, s>>>(segs, m, n, owner, W, H, 2 * (W + H) + 4 * 65536);
  const int npix = W * H;
  resolve_kernel<<<(npix + 255) / 256, 256, 0, s>>>(owner, colors, img, npix);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
