// Native host runtime of the autograd path (Python extension module _gsb_host)
// and the torch op namespace torch.ops.gsplat_b200 it registers.
//
// The ops allocate through the torch caching allocator, issue the C-ABI
// launches of include/gsplat_b200.h on the current stream and read the pair
// total once per forward (the only host sync, which the depth sort overlaps).
// rasterize_fwd drives a whole training or eval forward in one call and
// render_bwd a whole backward; bin / render_fwd_eval / render_fwd_train are the
// same steps one at a time. Native driving replaces op-by-op Python driving of
// the C entry points, whose interpreter overhead (~0.4 ms per fwd+bwd) was
// longer than the GPU work.
//
// Reference call sequence it drives (nbardy/fast-mac-gsplat):
//   _RasterizeProjectedGaussiansV8Project3D.forward/backward
//     variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:691-852
//   metal_bin + cumsum/.item()   variants/v8_project3d/csrc/metal/gsplat_metal.mm:317-379
#include <ATen/cuda/CUDAContext.h>
#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <array>
#include <cstdlib>
#include <map>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <tuple>
#include <string>
#include <vector>

#include "gsplat_b200.h"

namespace {

using at::Tensor;

void check(int rc, const char* what) {
  if (rc != GSB_OK)
    throw std::runtime_error(std::string(what) + " failed with status " + std::to_string(rc) + ": " +
                             gsb_status_string(rc));
}

std::string decode_device_error(uint32_t flags, uint32_t site) {
  std::string parts;
  auto add = [&](const char* s) { parts += (parts.empty() ? "" : "; ") + std::string(s); };
  if (flags & GSB_DEVERR_LOOKBACK_TIMEOUT) add("decoupled look-back wait exceeded its spin limit");
  if (flags & GSB_DEVERR_PAIR_OVERFLOW) add("pair count overflow (emit/scan mismatch or > 2^31 pairs)");
  if (flags & GSB_DEVERR_BOUNDS) add("index out of bounds");
  if (parts.empty()) parts = "unknown";
  return "gsplat_b200 device error (flags=" + std::to_string(flags) + ", site=" + std::to_string(site) + "): " +
         parts;
}

bool debug_checks() {
  const char* v = std::getenv("GSPLAT_B200_CHECK");
  return v != nullptr && v[0] != '\0' && !(v[0] == '0' && v[1] == '\0');
}

void* stream_of(const Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

template <typename T>
T* ptr(const Tensor& t) {
  return t.defined() ? static_cast<T*>(t.data_ptr()) : nullptr;
}

Tensor empty(at::IntArrayRef shape, at::ScalarType dt, const at::Device& dev) {
  return at::empty(shape, at::TensorOptions().dtype(dt).device(dev));
}

// Synchronous status read (debug checks, overflow check); raises on a device error.
std::array<uint32_t, GSB_STATUS_WORDS> read_status(const Tensor& status) {
  Tensor host = status.to(at::kCPU);  // blocks on the stream
  std::array<uint32_t, GSB_STATUS_WORDS> v{};
  const int32_t* p = host.data_ptr<int32_t>();
  for (int i = 0; i < GSB_STATUS_WORDS; ++i) v[i] = static_cast<uint32_t>(p[i]);
  if (v[GSB_STATUS_ERROR]) throw std::runtime_error(decode_device_error(v[GSB_STATUS_ERROR], v[GSB_STATUS_ERROR_SITE]));
  return v;
}

// The small device-to-host reads (the pair total, the deferred status copies)
// run on a side stream per device, ordered after the producing kernels by an
// event, so the compute stream never queues behind a copy.
c10::cuda::CUDAStream side_stream(c10::DeviceIndex dev) {
  static std::mutex mu;
  static std::map<int, c10::cuda::CUDAStream>* streams = new std::map<int, c10::cuda::CUDAStream>();
  std::lock_guard<std::mutex> g(mu);
  auto it = streams->find(dev);
  if (it == streams->end()) it = streams->emplace(dev, c10::cuda::getStreamFromPool(true, dev)).first;
  return it->second;
}

// Deferred device-error reads: each forward/backward queues a copy of its
// status block into a pinned slot on the side stream; the next forward (after
// its pair-count read, which follows every earlier copy on the side stream) or
// check_device_errors() reads them. Shared by all threads, because autograd
// runs backward on its own device thread.
struct ErrorRing {
  static constexpr int kSlots = 16;
  std::mutex mu;
  Tensor host;  // [kSlots, GSB_STATUS_WORDS] int32, pinned
  std::vector<at::cuda::CUDAEvent> events;  // copy done (side stream)
  std::vector<at::cuda::CUDAEvent> issued;  // status final (compute stream)
  std::array<cudaStream_t, kSlots> streams{};
  std::array<bool, kSlots> used{};
  int next = 0;

  void ensure() {
    if (!host.defined()) {
      host = at::empty({kSlots, GSB_STATUS_WORDS}, at::TensorOptions().dtype(at::kInt).pinned_memory(true));
      events.resize(kSlots);
      issued.resize(kSlots);
    }
  }
  // Caller holds mu.
  void check_slot(int i, cudaStream_t synced) {
    if (!used[i]) return;
    used[i] = false;
    if (streams[i] != synced) events[i].synchronize();
    const int32_t* p = host.data_ptr<int32_t>() + i * GSB_STATUS_WORDS;
    const uint32_t flags = static_cast<uint32_t>(p[GSB_STATUS_ERROR]);
    if (flags) throw std::runtime_error(decode_device_error(flags, static_cast<uint32_t>(p[GSB_STATUS_ERROR_SITE])));
  }
  void defer(const Tensor& status) {
    std::lock_guard<std::mutex> g(mu);
    ensure();
    const int i = next;
    next = (next + 1) % kSlots;
    check_slot(i, nullptr);
    const auto dev = status.device().index();
    auto cur = at::cuda::getCurrentCUDAStream(dev);
    auto side = side_stream(dev);
    issued[i].record(cur);
    issued[i].block(side);
    {
      const c10::cuda::CUDAStreamGuard sg(side);
      host[i].copy_(status, /*non_blocking=*/true);
    }
    status.record_stream(side);  // the allocator keeps it until the copy is done
    events[i].record(side);
    streams[i] = side.stream();
    used[i] = true;
  }
  void check_all(cudaStream_t synced) {
    std::lock_guard<std::mutex> g(mu);
    if (!host.defined()) return;
    for (int k = 0; k < kSlots; ++k) check_slot((next + k) % kSlots, synced);
  }
};
// Process-lifetime objects are created on first use and never destroyed: their
// destructors would call into CUDA and the torch allocator after those have
// been torn down at interpreter exit.
ErrorRing& errors() {
  static ErrorRing* r = new ErrorRing();
  return *r;
}

// Optional per-phase CUDA-event timing (bench instrumentation): events bracket
// each group of launches on the launching stream.
struct PhaseTimer {
  std::mutex mu;
  bool on = false;
  std::vector<std::pair<std::string, std::pair<at::cuda::CUDAEvent, at::cuda::CUDAEvent>>> marks;
};
PhaseTimer& phase_timer() {
  static PhaseTimer* t = new PhaseTimer();
  return *t;
}

struct Phase {
  at::cuda::CUDAEvent* end = nullptr;
  Phase(const char* name, const Tensor& like) {
    if (!phase_timer().on) return;
    PhaseTimer& pt = phase_timer();
    std::lock_guard<std::mutex> g(pt.mu);
    pt.marks.emplace_back(name, std::make_pair(at::cuda::CUDAEvent(cudaEventDefault),
                                               at::cuda::CUDAEvent(cudaEventDefault)));
    auto& pr = pt.marks.back().second;
    pr.first.record(at::cuda::getCurrentCUDAStream(like.device().index()));
    end = &pr.second;
    stream_index = like.device().index();
  }
  ~Phase() {
    if (end) end->record(at::cuda::getCurrentCUDAStream(stream_index));
  }
  int stream_index = 0;
};

gsb_raster_meta make_meta(int64_t H, int64_t W, int64_t B, int64_t G, double alpha_thr, double T_thr,
                          const std::vector<double>& bg, double eps, double max_alpha) {
  gsb_raster_meta m{};
  m.height = static_cast<int32_t>(H);
  m.width = static_cast<int32_t>(W);
  m.tile_size = 16;
  m.batch_size = static_cast<int32_t>(B);
  m.gaussians_per_batch = static_cast<int32_t>(G);
  m.alpha_threshold = static_cast<float>(alpha_thr);
  m.transmittance_threshold = static_cast<float>(T_thr);
  for (int c = 0; c < 3; ++c) m.background[c] = static_cast<float>(bg.at(c));
  m.eps = static_cast<float>(eps);
  m.max_alpha = static_cast<float>(max_alpha);
  return m;
}

Tensor aligned(const Tensor& t, int64_t align) {
  Tensor c = t.contiguous();
  if (reinterpret_cast<uintptr_t>(c.data_ptr()) % align) c = c.clone();
  return c;
}

// Pinned scalar for the pair total and the events that order its copy (on the
// side stream) after the count kernel.
struct PairRead {
  Tensor host;
  at::cuda::CUDAEvent counted;
  at::cuda::CUDAEvent done;
};
PairRead& pair_read() {
  thread_local PairRead* p = nullptr;
  if (p == nullptr) p = new PairRead();
  return *p;
}

// Scalar raster parameters shared by every op schema below (the reference
// packs the same values into its meta tensors, rasterize.py:109-141).
#define GSB_RASTER_ARGS                                                                                    \
  "int height, int width, float alpha_threshold, float transmittance_threshold, float bg_r, float bg_g, " \
  "float bg_b, float eps, float max_alpha"

// Argument errors surface in Python as ValueError (the reference's
// _check_inputs raises ValueError, …/rasterize.py:149-180).
[[noreturn]] void value_error(const std::string& msg) {
  TORCH_CHECK_VALUE(false, msg);
  throw std::logic_error(msg);  // not reached
}

void check_cuda_f32(const Tensor& t, const char* name) {
  if (!t.is_cuda()) value_error(std::string("gsplat_b200: ") + name + " must be a CUDA tensor");
  if (t.scalar_type() != at::kFloat) value_error(std::string("gsplat_b200: ") + name + " must be float32");
}

struct Binned {
  Tensor perm, rec, tile_offsets, binned_ids, status;
};

// Mean pairs per tile from which the tile ranges come from the last sort pass
// (gsb_bin_emit_ranges).
constexpr int64_t kFoldRangesMinPairsPerTile = 64;

// Depth sort, per-splat records and per-tile lists (reference: metal_bin +
// cumsum/.item(), …/gsplat_metal.mm:317-379; stable depth argsort and gathers,
// …/rasterize.py:708-717). pair_cap >= 0 raises the reference's overflow error
// when a tile holds more pairs than pair_cap (overflow fallback disabled); -1
// skips the check.
Binned bin_impl(const gsb_raster_meta& meta, const Tensor& means2d, const Tensor& conics, const Tensor& colors,
                const Tensor& opacities, const Tensor& depths, int64_t pair_cap) {
  const at::Device dev = means2d.device();
  const int64_t B = meta.batch_size, G = meta.gaussians_per_batch, BG = B * G;
  const int64_t H = meta.height, W = meta.width;
  void* stream = stream_of(means2d);
  const Tensor m2 = aligned(means2d, 8);
  const Tensor q2 = conics.contiguous(), c2 = colors.contiguous(), o2 = opacities.contiguous(),
               d2 = depths.contiguous();

  const size_t ws_bytes = gsb_bin_prepare_workspace_size(&meta);
  Binned r;
  r.status = empty({GSB_STATUS_WORDS}, at::kInt, dev);  // cleared by gsb_bin_count
  r.perm = empty({B, G}, at::kInt, dev);
  r.rec = empty({BG, GSB_REC_FLOATS}, at::kFloat, dev);
  Tensor pair_offsets = empty({BG + 1}, at::kInt, dev);
  // Hit masks / hit bits of each splat's candidate tiles (gsb_bin_tile_masks_size bytes).
  Tensor tile_masks = empty({static_cast<int64_t>((gsb_bin_tile_masks_size(&meta) + 7) / 8)}, at::kLong, dev);
  Tensor ws = empty({static_cast<int64_t>(std::max<size_t>(ws_bytes, 1))}, at::kByte, dev);
  auto cur = at::cuda::getCurrentCUDAStream(dev.index());
  PairRead& pr = pair_read();
  {
    Phase ph("bin_prepare", means2d);
    check(gsb_bin_count(&meta, ptr<float>(m2), ptr<float>(q2), ptr<float>(o2), ptr<float>(d2),
                        ptr<uint64_t>(tile_masks), ptr<uint32_t>(r.status), ws.data_ptr(), ws_bytes, stream),
          "gsb_bin_count");
    // The pair total is read on the side stream as soon as the count kernel is
    // done, while the depth sort and scan run on the compute stream.
    if (!pr.host.defined()) pr.host = at::empty({1}, at::TensorOptions().dtype(at::kLong).pinned_memory(true));
    auto side = side_stream(dev.index());
    pr.counted.record(cur);
    pr.counted.block(side);
    {
      const c10::cuda::CUDAStreamGuard sg(side);
      pr.host.copy_(r.status.narrow(0, GSB_STATUS_PAIR_TOTAL64, 2).view(at::kLong), /*non_blocking=*/true);
    }
    r.status.record_stream(side);
    pr.done.record(side);
    check(gsb_bin_sort_scan(&meta, ptr<float>(m2), ptr<float>(q2), ptr<float>(c2), ptr<float>(o2), ptr<float>(d2),
                            ptr<int32_t>(r.perm), ptr<float>(r.rec), ptr<int32_t>(pair_offsets),
                            ptr<uint64_t>(tile_masks), ptr<uint32_t>(r.status), ws.data_ptr(), ws_bytes, stream),
          "gsb_bin_sort_scan");
  }
  pr.done.synchronize();
  errors().check_all(side_stream(dev.index()).stream());  // every earlier copy on the side stream is complete now
  const int64_t P = pr.host.data_ptr<int64_t>()[0];
  if (P >= (int64_t(1) << 31) - 1)
    throw std::runtime_error("gsplat_b200: " + std::to_string(P) + " tile-splat pairs exceed the supported 2^31 - 1");
  const int64_t T = B * ((H + 15) / 16) * ((W + 15) / 16);
  const size_t ws2_bytes = gsb_bin_emit_workspace_size(&meta, P);
  r.binned_ids = empty({P}, at::kInt, dev);
  r.tile_offsets = empty({T + 1}, at::kInt, dev);
  Tensor ws2 = empty({static_cast<int64_t>(std::max<size_t>(ws2_bytes, 1))}, at::kByte, dev);
  {
    Phase ph("bin_emit", means2d);
    // Tile ranges from the last sort pass where tiles hold many pairs: it
    // saves 8 bytes per pair and costs a fixed amount per tile (c4, 7,300
    // pairs per tile: -60 us; c2, 57: +0.7 us; c3, 6: +2 us).
    if (P >= kFoldRangesMinPairsPerTile * T)
      check(gsb_bin_emit_ranges(&meta, ptr<float>(r.rec), ptr<int32_t>(pair_offsets), ptr<uint64_t>(tile_masks), P,
                                ptr<int32_t>(r.binned_ids), ptr<int32_t>(r.tile_offsets), ptr<uint32_t>(r.status),
                                ws2.data_ptr(), ws2_bytes, stream),
            "gsb_bin_emit_ranges");
    else
      check(gsb_bin_emit(&meta, ptr<float>(r.rec), ptr<int32_t>(pair_offsets), ptr<uint64_t>(tile_masks), P,
                         /*keys=*/nullptr, ptr<int32_t>(r.binned_ids), ptr<int32_t>(r.tile_offsets),
                         ptr<uint32_t>(r.status), ws2.data_ptr(), ws2_bytes, stream),
            "gsb_bin_emit");
  }
  if (debug_checks()) read_status(r.status);
  if (pair_cap >= 0) {
    check(gsb_tile_stats(&meta, ptr<int32_t>(r.tile_offsets), ptr<uint32_t>(r.status), stream), "gsb_tile_stats");
    const auto v = read_status(r.status);
    if (static_cast<int64_t>(v[GSB_STATUS_MAX_TILE_COUNT]) > pair_cap)
      throw std::runtime_error("Tile overflow detected with max_fast_pairs=" + std::to_string(pair_cap) +
                               ". Enable overflow fallback or increase the runtime cap.");
  }
  return r;
}

// Compositing forward (reference: tile_fast_forward_eval / _state,
// …/gsplat_v8_project3d_kernels.metal:783-929). save_state adds the per-pixel
// final transmittance, last-contributor count and the list-ordered record copy
// the backward reads. The status block's device errors are checked later
// (deferred), or now under GSPLAT_B200_CHECK.
std::vector<Tensor> render_fwd_impl(const gsb_raster_meta& meta, const Tensor& rec, const Tensor& tile_offsets,
                                    const Tensor& binned_ids, const Tensor& status, bool save_state) {
  const at::Device dev = rec.device();
  const int64_t B = meta.batch_size, H = meta.height, W = meta.width;
  const int64_t P = binned_ids.numel();
  void* stream = stream_of(rec);
  Tensor out = empty({B, H, W, 3}, at::kFloat, dev);
  Tensor final_T, last_idx, pair_rec;
  if (save_state) {
    final_T = empty({B, H, W}, at::kFloat, dev);
    last_idx = empty({B, H, W}, at::kInt, dev);
    pair_rec = empty({std::max<int64_t>(P, 1), GSB_REC_FLOATS}, at::kFloat, dev);
  }
  const size_t rws_bytes = gsb_render_workspace_size(&meta);
  Tensor rws = empty({static_cast<int64_t>(std::max<size_t>(rws_bytes, 1))}, at::kByte, dev);
  {
    Phase ph("render_fwd", rec);
    check(gsb_render_forward(&meta, ptr<float>(rec), ptr<int32_t>(tile_offsets), ptr<int32_t>(binned_ids),
                             ptr<float>(out), ptr<float>(final_T), ptr<int32_t>(last_idx), ptr<float>(pair_rec),
                             ptr<uint32_t>(status), rws.data_ptr(), rws_bytes, stream),
          "gsb_render_forward");
  }
  if (debug_checks())
    read_status(status);
  else
    errors().defer(status);
  if (!save_state) return {out};
  return {out, final_T, last_idx, pair_rec};
}

// Reverse-order VJP and un-sort into input order (reference:
// tile_fast_backward_saved, …/gsplat_v8_project3d_kernels.metal:931-1063;
// _unsort_batched, …/rasterize.py:583-591). From 2^18 splats the un-sort is
// folded into the backward's atomics (gsb_render_backward_inputs), which then
// target slices of one zeroed buffer; below, the atomics go to packed records
// in rank order and gsb_unsort_grads scatters them: there the input-order
// targets (four arrays, at permuted positions) cost the backward more L2
// traffic than the un-sort launch it saves (c3: +40 us against 11 us), while
// at 2^20 splats the un-sort is the dearer part (c4: -60 us). Gradients
// whose needs flag is false come back undefined (None in Python).
constexpr int64_t kFoldUnsortMinSplats = int64_t(1) << 18;

std::tuple<Tensor, Tensor, Tensor, Tensor> render_bwd_impl(const gsb_raster_meta& meta, const Tensor& perm,
                                                           const Tensor& rec, const Tensor& tile_offsets,
                                                           const Tensor& binned_ids, const Tensor& final_T,
                                                           const Tensor& last_idx, const Tensor& pair_rec,
                                                           const Tensor& status, const Tensor& grad_out,
                                                           std::array<bool, 4> needs) {
  const at::Device dev = rec.device();
  const int64_t B = meta.batch_size, G = meta.gaussians_per_batch;
  void* stream = stream_of(rec);
  const Tensor g = aligned(grad_out.to(at::kFloat), 16);
  const int64_t BG = B * G;
  if (BG < kFoldUnsortMinSplats) {
    const size_t ws_bytes = gsb_render_workspace_size(&meta);
    Tensor grad_rec = empty({BG, GSB_REC_FLOATS}, at::kFloat, dev);
    Tensor ws = empty({static_cast<int64_t>(std::max<size_t>(ws_bytes, 1))}, at::kByte, dev);
    {
      Phase ph("render_bwd", rec);
      check(gsb_render_backward(&meta, ptr<float>(rec), ptr<int32_t>(tile_offsets), ptr<int32_t>(binned_ids),
                                ptr<float>(final_T), ptr<int32_t>(last_idx), ptr<float>(pair_rec), ptr<float>(g),
                                ptr<float>(grad_rec), ptr<uint32_t>(status), ws.data_ptr(), ws_bytes, stream),
            "gsb_render_backward");
    }
    Tensor gm, gc, gcol, go;
    if (needs[0]) gm = empty({B, G, 2}, at::kFloat, dev);
    if (needs[1]) gc = empty({B, G, 3}, at::kFloat, dev);
    if (needs[2]) gcol = empty({B, G, 3}, at::kFloat, dev);
    if (needs[3]) go = empty({B, G}, at::kFloat, dev);
    {
      Phase ph("unsort", rec);
      check(gsb_unsort_grads(&meta, ptr<int32_t>(perm), ptr<float>(grad_rec), ptr<float>(gm), ptr<float>(gc),
                             ptr<float>(gcol), ptr<float>(go), stream),
            "gsb_unsort_grads");
    }
    if (debug_checks())
      read_status(status);
    else
      errors().defer(status);
    return {gm, gc, gcol, go};
  }
  // Slices of one buffer, in the order means2d (2), conics (3), colours (3),
  // opacities (1) floats per splat, only for the requested gradients.
  const int64_t widths[4] = {2, 3, 3, 1};
  int64_t floats = 0;
  for (int i = 0; i < 4; ++i) floats += needs[i] ? widths[i] * BG : 0;
  Tensor buf = at::zeros({std::max<int64_t>(floats, 1)}, at::TensorOptions().dtype(at::kFloat).device(dev));
  Tensor gm, gc, gcol, go;
  int64_t off = 0;
  auto take = [&](int i, std::vector<int64_t> shape) {
    Tensor t = buf.narrow(0, off, widths[i] * BG).view(shape);
    off += widths[i] * BG;
    return t;
  };
  if (needs[0]) gm = take(0, {B, G, 2});
  if (needs[1]) gc = take(1, {B, G, 3});
  if (needs[2]) gcol = take(2, {B, G, 3});
  if (needs[3]) go = take(3, {B, G});
  {
    Phase ph("render_bwd", rec);
    check(gsb_render_backward_inputs(&meta, ptr<float>(rec), ptr<int32_t>(tile_offsets), ptr<int32_t>(binned_ids),
                                     ptr<float>(final_T), ptr<int32_t>(last_idx), ptr<float>(pair_rec), ptr<float>(g),
                                     ptr<int32_t>(perm), ptr<float>(gm), ptr<float>(gc), ptr<float>(gcol),
                                     ptr<float>(go), ptr<uint32_t>(status), stream),
          "gsb_render_backward_inputs");
  }
  if (debug_checks())
    read_status(status);
  else
    errors().defer(status);
  return {gm, gc, gcol, go};
}

// ---- torch.ops.gsplat_b200 kernels (CUDA dispatch key) --------------------

void check_2d_inputs(const Tensor& means2d, const Tensor& conics, const Tensor& colors, const Tensor& opacities,
                     const Tensor& depths) {
  check_cuda_f32(means2d, "means2d");
  check_cuda_f32(conics, "conics");
  check_cuda_f32(colors, "colors");
  check_cuda_f32(opacities, "opacities");
  check_cuda_f32(depths, "depths");
  if (means2d.dim() != 3 || means2d.size(2) != 2) value_error("gsplat_b200: means2d must be [B,G,2]");
  const int64_t B = means2d.size(0), G = means2d.size(1);
  auto want = [&](const Tensor& t, int64_t last, const char* name) {
    const bool ok = last > 0 ? (t.dim() == 3 && t.size(0) == B && t.size(1) == G && t.size(2) == last)
                             : (t.dim() == 2 && t.size(0) == B && t.size(1) == G);
    if (!ok) value_error(std::string("gsplat_b200: ") + name + " shape does not match means2d [B,G]");
  };
  want(conics, 3, "conics");
  want(colors, 3, "colors");
  want(opacities, 0, "opacities");
  want(depths, 0, "depths");
}

gsb_raster_meta meta_of(int64_t B, int64_t G, int64_t H, int64_t W, double alpha_thr, double T_thr, double bg_r,
                        double bg_g, double bg_b, double eps, double max_alpha) {
  return make_meta(H, W, B, G, alpha_thr, T_thr, {bg_r, bg_g, bg_b}, eps, max_alpha);
}

int64_t gaussians_of(const Tensor& rec, int64_t B) {
  if (B <= 0 || rec.dim() != 2 || rec.size(0) % B != 0)
    value_error("gsplat_b200: rec must be [B*G, 12] for the given batch_size");
  return rec.size(0) / B;
}

// One-call forward: bin + render. Returns [image] (save_state false) or
// [image, perm, rec, tile_offsets, binned_ids, final_T, last_idx, pair_rec, status].
std::vector<Tensor> op_rasterize_fwd(const Tensor& means2d, const Tensor& conics, const Tensor& colors,
                                     const Tensor& opacities, const Tensor& depths, int64_t H, int64_t W,
                                     double alpha_thr, double T_thr, double bg_r, double bg_g, double bg_b, double eps,
                                     double max_alpha, bool save_state, int64_t pair_cap) {
  check_2d_inputs(means2d, conics, colors, opacities, depths);
  const c10::cuda::CUDAGuard guard(means2d.device());
  const gsb_raster_meta meta =
      meta_of(means2d.size(0), means2d.size(1), H, W, alpha_thr, T_thr, bg_r, bg_g, bg_b, eps, max_alpha);
  Binned b = bin_impl(meta, means2d, conics, colors, opacities, depths, pair_cap);
  std::vector<Tensor> r = render_fwd_impl(meta, b.rec, b.tile_offsets, b.binned_ids, b.status, save_state);
  if (!save_state) return r;
  return {r[0], b.perm, b.rec, b.tile_offsets, b.binned_ids, r[1], r[2], r[3], b.status};
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> op_bin(const Tensor& means2d, const Tensor& conics,
                                                          const Tensor& colors, const Tensor& opacities,
                                                          const Tensor& depths, int64_t H, int64_t W,
                                                          double alpha_thr, double T_thr, double bg_r, double bg_g,
                                                          double bg_b, double eps, double max_alpha,
                                                          int64_t pair_cap) {
  check_2d_inputs(means2d, conics, colors, opacities, depths);
  const c10::cuda::CUDAGuard guard(means2d.device());
  const gsb_raster_meta meta =
      meta_of(means2d.size(0), means2d.size(1), H, W, alpha_thr, T_thr, bg_r, bg_g, bg_b, eps, max_alpha);
  Binned b = bin_impl(meta, means2d, conics, colors, opacities, depths, pair_cap);
  if (!debug_checks()) errors().defer(b.status);
  return {b.perm, b.rec, b.tile_offsets, b.binned_ids, b.status};
}

Tensor op_render_fwd_eval(const Tensor& rec, const Tensor& tile_offsets, const Tensor& binned_ids,
                          const Tensor& status, int64_t B, int64_t H, int64_t W, double alpha_thr, double T_thr,
                          double bg_r, double bg_g, double bg_b, double eps, double max_alpha) {
  check_cuda_f32(rec, "rec");
  const c10::cuda::CUDAGuard guard(rec.device());
  const gsb_raster_meta meta =
      meta_of(B, gaussians_of(rec, B), H, W, alpha_thr, T_thr, bg_r, bg_g, bg_b, eps, max_alpha);
  return render_fwd_impl(meta, rec, tile_offsets, binned_ids, status, false)[0];
}

std::tuple<Tensor, Tensor, Tensor, Tensor> op_render_fwd_train(const Tensor& rec, const Tensor& tile_offsets,
                                                               const Tensor& binned_ids, const Tensor& status,
                                                               int64_t B, int64_t H, int64_t W, double alpha_thr,
                                                               double T_thr, double bg_r, double bg_g, double bg_b,
                                                               double eps, double max_alpha) {
  check_cuda_f32(rec, "rec");
  const c10::cuda::CUDAGuard guard(rec.device());
  const gsb_raster_meta meta =
      meta_of(B, gaussians_of(rec, B), H, W, alpha_thr, T_thr, bg_r, bg_g, bg_b, eps, max_alpha);
  std::vector<Tensor> r = render_fwd_impl(meta, rec, tile_offsets, binned_ids, status, true);
  return {r[0], r[1], r[2], r[3]};
}

std::tuple<Tensor, Tensor, Tensor, Tensor> op_render_bwd(const Tensor& perm, const Tensor& rec,
                                                         const Tensor& tile_offsets, const Tensor& binned_ids,
                                                         const Tensor& final_T, const Tensor& last_idx,
                                                         const Tensor& pair_rec, const Tensor& status,
                                                         const Tensor& grad_image, int64_t H, int64_t W,
                                                         double alpha_thr, double T_thr, double bg_r, double bg_g,
                                                         double bg_b, double eps, double max_alpha,
                                                         std::array<bool, 4> needs) {
  if (perm.dim() != 2) value_error("gsplat_b200: perm must be [B,G]");
  if (grad_image.dim() != 4 || grad_image.size(0) != perm.size(0) || grad_image.size(1) != H ||
      grad_image.size(2) != W || grad_image.size(3) != 3)
    value_error("gsplat_b200: grad_image must be [B,H,W,3]");
  const c10::cuda::CUDAGuard guard(rec.device());
  const gsb_raster_meta meta =
      meta_of(perm.size(0), perm.size(1), H, W, alpha_thr, T_thr, bg_r, bg_g, bg_b, eps, max_alpha);
  return render_bwd_impl(meta, perm, rec, tile_offsets, binned_ids, final_T, last_idx, pair_rec, status, grad_image,
                         needs);
}

void check_3d_inputs(const Tensor& means3d, const Tensor& scales, const Tensor& quats, const Tensor& opacities,
                     const Tensor& c2w, const Tensor& cam) {
  check_cuda_f32(means3d, "means3d");
  check_cuda_f32(scales, "scales");
  check_cuda_f32(quats, "quats");
  check_cuda_f32(opacities, "opacities");
  check_cuda_f32(c2w, "camera_to_world");
  check_cuda_f32(cam, "camera_params");
  if (means3d.dim() != 3 || means3d.size(2) != 3) value_error("gsplat_b200: means3d must be [B,G,3]");
  const int64_t B = means3d.size(0), G = means3d.size(1);
  if (scales.sizes() != means3d.sizes()) value_error("gsplat_b200: scales must be [B,G,3]");
  if (quats.dim() != 3 || quats.size(0) != B || quats.size(1) != G || quats.size(2) != 4)
    value_error("gsplat_b200: quats must be [B,G,4]");
  if (opacities.dim() != 2 || opacities.size(0) != B || opacities.size(1) != G)
    value_error("gsplat_b200: opacities must be [B,G]");
  if (c2w.dim() != 3 || c2w.size(0) != B || c2w.size(1) != 4 || c2w.size(2) != 4)
    value_error("gsplat_b200: camera_to_world must be [B,4,4]");
  if (cam.dim() != 2 || cam.size(0) != B || cam.size(1) != 4)
    value_error("gsplat_b200: camera_params must be [B,4]");
}

// Pinhole projection (reference: project_pinhole_forward,
// …/gsplat_v8_project3d_kernels.metal:66-174) -> means2d, conics, opacities, depths.
std::tuple<Tensor, Tensor, Tensor, Tensor> op_project_fwd(const Tensor& means3d, const Tensor& scales,
                                                          const Tensor& quats, const Tensor& opacities,
                                                          const Tensor& c2w, const Tensor& cam, double near_plane) {
  check_3d_inputs(means3d, scales, quats, opacities, c2w, cam);
  const c10::cuda::CUDAGuard guard(means3d.device());
  const at::Device dev = means3d.device();
  const int64_t B = means3d.size(0), G = means3d.size(1);
  Tensor om = empty({B, G, 2}, at::kFloat, dev), oc = empty({B, G, 3}, at::kFloat, dev);
  Tensor oo = empty({B, G}, at::kFloat, dev), od = empty({B, G}, at::kFloat, dev);
  const Tensor m3 = means3d.contiguous(), s3 = scales.contiguous(), o1 = opacities.contiguous();
  const Tensor q4 = aligned(quats, 16), k16 = aligned(c2w, 16), k4 = aligned(cam, 16);
  check(gsb_project_forward(static_cast<int32_t>(B), static_cast<int32_t>(G), ptr<float>(m3), ptr<float>(s3),
                            ptr<float>(q4), ptr<float>(o1), ptr<float>(k16), ptr<float>(k4),
                            static_cast<float>(near_plane), ptr<float>(om), ptr<float>(oc), ptr<float>(oo),
                            ptr<float>(od), stream_of(means3d)),
        "gsb_project_forward");
  return {om, oc, oo, od};
}

Tensor opt_grad(const std::optional<Tensor>& g) {
  if (!g.has_value() || !g->defined()) return Tensor();
  return aligned(g->to(at::kFloat), 16);
}

// Projection VJP (reference: project_pinhole_backward,
// …/gsplat_v8_project3d_kernels.metal:217-501); absent incoming gradients are
// zeros. -> g_means3d, g_scales, g_quats, g_opacities, g_camera_to_world, g_camera_params.
std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> op_project_bwd(
    const std::optional<Tensor>& g_m2d, const std::optional<Tensor>& g_con, const std::optional<Tensor>& g_op,
    const std::optional<Tensor>& g_depth, const Tensor& means3d, const Tensor& scales, const Tensor& quats,
    const Tensor& opacities, const Tensor& c2w, const Tensor& cam, double near_plane) {
  check_3d_inputs(means3d, scales, quats, opacities, c2w, cam);
  const c10::cuda::CUDAGuard guard(means3d.device());
  const at::Device dev = means3d.device();
  const int64_t B = means3d.size(0), G = means3d.size(1);
  const Tensor gm2 = opt_grad(g_m2d), gco = opt_grad(g_con), gop = opt_grad(g_op), gde = opt_grad(g_depth);
  Tensor gm3 = empty({B, G, 3}, at::kFloat, dev), gs = empty({B, G, 3}, at::kFloat, dev);
  Tensor gq = empty({B, G, 4}, at::kFloat, dev), go = empty({B, G}, at::kFloat, dev);
  Tensor gc2w = empty({B, 4, 4}, at::kFloat, dev), gcam = empty({B, 4}, at::kFloat, dev);
  const Tensor m3 = means3d.contiguous(), s3 = scales.contiguous(), o1 = opacities.contiguous();
  const Tensor q4 = aligned(quats, 16), k16 = aligned(c2w, 16), k4 = aligned(cam, 16);
  check(gsb_project_backward(static_cast<int32_t>(B), static_cast<int32_t>(G), ptr<float>(gm2), ptr<float>(gco),
                             ptr<float>(gop), ptr<float>(gde), ptr<float>(m3), ptr<float>(s3), ptr<float>(q4),
                             ptr<float>(o1), ptr<float>(k16), ptr<float>(k4), static_cast<float>(near_plane),
                             ptr<float>(gm3), ptr<float>(gs), ptr<float>(gq), ptr<float>(go), ptr<float>(gc2w),
                             ptr<float>(gcam), stream_of(means3d)),
        "gsb_project_backward");
  return {gm3, gs, gq, go, gc2w, gcam};
}

void check_sh_inputs(const Tensor& sh, const Tensor& means3d, const Tensor& c2w, int64_t degree) {
  check_cuda_f32(sh, "sh_coeffs");
  check_cuda_f32(means3d, "means3d");
  check_cuda_f32(c2w, "camera_to_world");
  if (degree < 0 || degree > 3) value_error("gsplat_b200: SH degree must be 0..3");
  const int64_t K = (degree + 1) * (degree + 1);
  if (sh.dim() != 3 || sh.size(1) != K || sh.size(2) != 3)
    value_error("gsplat_b200: sh_coeffs must be [G,(degree+1)^2,3]");
  if (means3d.dim() != 2 || means3d.size(0) != sh.size(0) || means3d.size(1) != 3)
    value_error("gsplat_b200: means3d must be [G,3]");
  if (c2w.dim() != 3 || c2w.size(1) != 4 || c2w.size(2) != 4)
    value_error("gsplat_b200: camera_to_world must be [B,4,4]");
}

// View-dependent colours from SH coefficients (no reference counterpart; the
// reference's 3D entry point takes RGB colours) -> colors [B,G,3].
Tensor op_sh_fwd(const Tensor& sh, const Tensor& means3d, const Tensor& c2w, int64_t degree) {
  check_sh_inputs(sh, means3d, c2w, degree);
  const c10::cuda::CUDAGuard guard(sh.device());
  const int64_t B = c2w.size(0), G = means3d.size(0);
  const Tensor s = sh.contiguous(), m = means3d.contiguous(), k = c2w.contiguous();
  Tensor colors = empty({B, G, 3}, at::kFloat, sh.device());
  check(gsb_sh_forward(static_cast<int32_t>(B), static_cast<int32_t>(G), static_cast<int32_t>(degree), ptr<float>(s),
                       ptr<float>(m), ptr<float>(k), ptr<float>(colors), stream_of(sh)),
        "gsb_sh_forward");
  return colors;
}

std::tuple<Tensor, Tensor, Tensor> op_sh_bwd(const Tensor& sh, const Tensor& means3d, const Tensor& c2w,
                                             const Tensor& colors, const Tensor& grad_colors, int64_t degree,
                                             bool need_means3d, bool need_c2w) {
  check_sh_inputs(sh, means3d, c2w, degree);
  const c10::cuda::CUDAGuard guard(sh.device());
  const at::Device dev = sh.device();
  const int64_t B = c2w.size(0), G = means3d.size(0);
  const Tensor s = sh.contiguous(), m = means3d.contiguous(), k = c2w.contiguous(), c = colors.contiguous();
  const Tensor g = grad_colors.to(at::kFloat).contiguous();
  Tensor g_sh = at::empty_like(s);
  Tensor g_m = need_means3d ? empty({G, 3}, at::kFloat, dev) : Tensor();
  Tensor g_k = need_c2w ? empty({B, 4, 4}, at::kFloat, dev) : Tensor();
  check(gsb_sh_backward(static_cast<int32_t>(B), static_cast<int32_t>(G), static_cast<int32_t>(degree), ptr<float>(s),
                        ptr<float>(m), ptr<float>(k), ptr<float>(c), ptr<float>(g), ptr<float>(g_sh), ptr<float>(g_m),
                        ptr<float>(g_k), stream_of(sh)),
        "gsb_sh_backward");
  return {g_sh, g_m, g_k};
}

void check_device_errors() { errors().check_all(nullptr); }

void set_phase_timing(bool on) {
  std::lock_guard<std::mutex> g(phase_timer().mu);
  phase_timer().on = on;
  phase_timer().marks.clear();
}

// Elapsed milliseconds of every timed phase since set_phase_timing(true)
// (synchronizes on the recorded events), then clears the record.
std::map<std::string, std::vector<double>> take_phase_times() {
  std::lock_guard<std::mutex> g(phase_timer().mu);
  std::map<std::string, std::vector<double>> out;
  for (auto& mk : phase_timer().marks) {
    mk.second.second.synchronize();
    out[mk.first].push_back(mk.second.first.elapsed_time(mk.second.second));
  }
  phase_timer().marks.clear();
  return out;
}

}  // namespace

// Reference op namespace: gsplat_metal_v8_project3d.{bin, project_pinhole_forward,
// project_pinhole_backward, render_fast_forward_eval, render_fast_forward_state,
// render_fast_backward_saved} (variants/v8_project3d/csrc/bindings.cpp:173-193),
// there registered for CompositeExplicitAutograd on MPS tensors; here for the
// CUDA dispatch key only, so CPU tensors raise instead of falling back.
TORCH_LIBRARY(gsplat_b200, m) {
  m.def("rasterize_fwd(Tensor means2d, Tensor conics, Tensor colors, Tensor opacities, Tensor depths, " GSB_RASTER_ARGS
        ", bool save_state, int pair_cap) -> Tensor[]");
  m.def("bin(Tensor means2d, Tensor conics, Tensor colors, Tensor opacities, Tensor depths, " GSB_RASTER_ARGS
        ", int pair_cap) -> (Tensor perm, Tensor rec, Tensor tile_offsets, Tensor binned_ids, Tensor status)");
  m.def("render_fwd_eval(Tensor rec, Tensor tile_offsets, Tensor binned_ids, Tensor(a!) status, int batch_size, "
        GSB_RASTER_ARGS ") -> Tensor");
  m.def("render_fwd_train(Tensor rec, Tensor tile_offsets, Tensor binned_ids, Tensor(a!) status, int batch_size, "
        GSB_RASTER_ARGS ") -> (Tensor image, Tensor final_T, Tensor last_idx, Tensor pair_rec)");
  m.def("render_bwd(Tensor perm, Tensor rec, Tensor tile_offsets, Tensor binned_ids, Tensor final_T, "
        "Tensor last_idx, Tensor pair_rec, Tensor(a!) status, Tensor grad_image, " GSB_RASTER_ARGS
        ", bool[4] needs) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("project_fwd(Tensor means3d, Tensor scales, Tensor quats, Tensor opacities, Tensor camera_to_world, "
        "Tensor camera_params, float near_plane) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("project_bwd(Tensor? grad_means2d, Tensor? grad_conics, Tensor? grad_opacities, Tensor? grad_depths, "
        "Tensor means3d, Tensor scales, Tensor quats, Tensor opacities, Tensor camera_to_world, "
        "Tensor camera_params, float near_plane) -> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("sh_fwd(Tensor sh_coeffs, Tensor means3d, Tensor camera_to_world, int degree) -> Tensor");
  m.def("sh_bwd(Tensor sh_coeffs, Tensor means3d, Tensor camera_to_world, Tensor colors, Tensor grad_colors, "
        "int degree, bool need_means3d, bool need_camera_to_world) -> (Tensor, Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(gsplat_b200, CUDA, m) {
  m.impl("rasterize_fwd", &op_rasterize_fwd);
  m.impl("bin", &op_bin);
  m.impl("render_fwd_eval", &op_render_fwd_eval);
  m.impl("render_fwd_train", &op_render_fwd_train);
  m.impl("render_bwd", &op_render_bwd);
  m.impl("project_fwd", &op_project_fwd);
  m.impl("project_bwd", &op_project_bwd);
  m.impl("sh_fwd", &op_sh_fwd);
  m.impl("sh_bwd", &op_sh_bwd);
}

PYBIND11_MODULE(_gsb_host, m) {
  m.doc() = "Native host runtime of the B200 rasterizer autograd path (drives the C ABI).";
  m.def("check_device_errors", &check_device_errors);
  m.def("set_phase_timing", &set_phase_timing);
  m.def("take_phase_times", &take_phase_times);
}
