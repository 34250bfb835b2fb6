// Headless isometric voxel rasteriser for the liveSee project.
//
// The reference draws its view in the browser with canvas-2D (painter's
// order over cubes sorted by x+y+z, three shaded quads per cube,
// project/liveSee/play_live_world.py).  Here the same picture is produced on
// the GPU into an RGBA8 device buffer:
//   pass 1  one CTA per quad: every pixel centre of the quad's bounding box
//           that lies inside the convex quad (edge functions, double
//           precision) takes atomicMax(draw order + 1) -- the quad drawn last
//           by the painter's algorithm wins, exactly as overdraw would;
//   pass 2  one thread per pixel resolves the winning quad's colour or the
//           sky / ground background.
// The host passes quads already projected and sorted (draw order = index).
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace uhfs {

namespace {

__device__ __forceinline__ double edge(double ax, double ay, double bx, double by, double px, double py) {
  return (bx - ax) * (py - ay) - (by - ay) * (px - ax);
}

__global__ void raster_cover_kernel(const float* __restrict__ quads, int nquads, unsigned int* __restrict__ order,
                                    int width, int height) {
  const int q = blockIdx.x;
  if (q >= nquads) return;
  const float* p = quads + q * 8;  // x0 y0 x1 y1 x2 y2 x3 y3
  float minx = p[0], maxx = p[0], miny = p[1], maxy = p[1];
  for (int i = 1; i < 4; ++i) {
    minx = fminf(minx, p[2 * i]);
    maxx = fmaxf(maxx, p[2 * i]);
    miny = fminf(miny, p[2 * i + 1]);
    maxy = fmaxf(maxy, p[2 * i + 1]);
  }
  const int x0 = max(0, (int)floorf(minx)), x1 = min(width - 1, (int)ceilf(maxx));
  const int y0 = max(0, (int)floorf(miny)), y1 = min(height - 1, (int)ceilf(maxy));
  if (x0 > x1 || y0 > y1) return;
  const int bw = x1 - x0 + 1, bh = y1 - y0 + 1;
  for (int i = threadIdx.x; i < bw * bh; i += blockDim.x) {
    const double px = x0 + i % bw + 0.5, py = y0 + i / bw + 0.5;
    bool pos = true, neg = true;
    for (int e = 0; e < 4; ++e) {
      const int f = (e + 1) & 3;
      const double v = edge(p[2 * e], p[2 * e + 1], p[2 * f], p[2 * f + 1], px, py);
      pos = pos && v >= 0.0;
      neg = neg && v <= 0.0;
    }
    if (pos || neg) atomicMax(order + (y0 + i / bw) * width + (x0 + i % bw), (unsigned int)(q + 1));
  }
}

__global__ void raster_resolve_kernel(const unsigned int* __restrict__ order, const unsigned int* __restrict__ colors,
                                      unsigned int* __restrict__ rgba, int width, int height) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= width * height) return;
  const unsigned int o = order[idx];
  if (o != 0u) {
    rgba[idx] = colors[o - 1];
    return;
  }
  // background: #78c7ff -> #d8f6ff down to 52% of the height, #222222 below
  const int y = idx / width;
  const float t = (y + 0.5f) / (float)height;
  unsigned int r, g, b;
  if (t < 0.52f) {
    const float u = t / 0.52f;
    r = (unsigned int)(0x78 + (0xd8 - 0x78) * u + 0.5f);
    g = (unsigned int)(0xc7 + (0xf6 - 0xc7) * u + 0.5f);
    b = (unsigned int)(0xff + (0xff - 0xff) * u + 0.5f);
  } else {
    r = g = b = 0x22;
  }
  rgba[idx] = r | (g << 8) | (b << 16) | (0xffu << 24);
}

}  // namespace

void raster_iso(const float* quads, const unsigned int* colors, int nquads, unsigned int* order, unsigned int* rgba,
                int width, int height, cudaStream_t s) {
  UHFS_CUDA_CHECK(cudaMemsetAsync(order, 0, (size_t)width * height * sizeof(unsigned int), s));
  if (nquads > 0) {
    raster_cover_kernel<<<nquads, 256, 0, s>>>(quads, nquads, order, width, height);
    note_launch();
  }
  raster_resolve_kernel<<<(width * height + 255) / 256, 256, 0, s>>>(order, colors, rgba, width, height);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace uhfs
