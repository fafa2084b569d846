// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>

#include "gsb_common.cuh"

namespace gsb {

// Bump allocator over a caller-provided workspace. With base == nullptr it only
// measures (the *_workspace_size queries run the same carve sequence).
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

// Process-wide count of kernel launches issued by this library.
void note_launches(uint64_t n);

// Magic numbers of fast_div for a divisor 1 <= d < 2^31 (d = 0 is taken as 1).
inline FastDiv make_fast_div(uint32_t d) {
  FastDiv f;
  if (d == 0) d = 1;
  uint32_t l = 0;
  while ((uint64_t(1) << l) < d) ++l;
  f.shift = l;
  f.mul = (uint32_t)(((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1);
  return f;
}

// Validates a gsb_raster_meta and expands it into the kernel-side Meta.
inline int make_meta(const gsb_raster_meta* in, Meta* m) {
  if (in == nullptr || m == nullptr) return GSB_ERR_INVALID_ARGUMENT;
  if (in->tile_size != kTile) return GSB_ERR_UNSUPPORTED;
  if (in->height <= 0 || in->width <= 0 || in->batch_size <= 0 || in->gaussians_per_batch < 0)
    return GSB_ERR_INVALID_ARGUMENT;
  const int64_t tiles_x = (in->width + kTile - 1) / kTile;
  const int64_t tiles_y = (in->height + kTile - 1) / kTile;
  const int64_t tpi = tiles_x * tiles_y;
  const int64_t total_tiles = tpi * in->batch_size;
  const int64_t bg = (int64_t)in->batch_size * in->gaussians_per_batch;
  const int64_t pixels = (int64_t)in->batch_size * in->height * in->width;
  if (total_tiles >= (int64_t(1) << 31) - 1 || bg >= (int64_t(1) << 31) - 1 || pixels >= (int64_t(1) << 40))
    return GSB_ERR_INVALID_ARGUMENT;
  m->H = in->height;
  m->W = in->width;
  m->tiles_x = (int)tiles_x;
  m->tiles_y = (int)tiles_y;
  m->tiles_per_image = (int)tpi;
  m->B = in->batch_size;
  m->G = in->gaussians_per_batch;
  m->BG = (int)bg;
  m->total_tiles = (int)total_tiles;
  m->alpha_thr = in->alpha_threshold;
  m->T_thr = in->transmittance_threshold;
  m->bg_r = in->background[0];
  m->bg_g = in->background[1];
  m->bg_b = in->background[2];
  m->eps = in->eps;
  m->max_alpha = in->max_alpha;
  m->div_tiles_x = make_fast_div((uint32_t)tiles_x);
  m->div_tiles_per_image = make_fast_div((uint32_t)tpi);
  m->div_G = make_fast_div(in->gaussians_per_batch > 0 ? (uint32_t)in->gaussians_per_batch : 1u);
  return GSB_OK;
}

inline int bits_for(int64_t max_value) {
  int b = 0;
  while (b < 63 && (int64_t(1) << b) <= max_value) ++b;
  return b;
}

inline int grid1d(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  return (int)(b < 1 ? 1 : b);
}

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? GSB_OK : GSB_ERR_CUDA; }

// Launches a kernel of this library with programmatic stream serialization
// (the kernel starts with pdl_wait / pdl_trigger, see gsb_common.cuh).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
  static_assert(sizeof...(KArgs) == sizeof...(Args), "kernel argument count");
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}


}  // namespace gsb
