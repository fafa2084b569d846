// Native host runtime of the autograd path (Python extension module _gsb_host).
//
// One call drives a whole training or eval forward and one call a whole
// backward: it allocates through the torch caching allocator, issues the C-ABI
// launches of include/gsplat_b200.h on the current stream, and reads the pair
// total once (the only host sync of a forward, which the depth sort overlaps).
// It replaces the op-by-op Python driving of the same C entry points, whose
// interpreter overhead (~0.4 ms per fwd+bwd) was longer than the GPU work.
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

// Deferred device-error reads: each forward/backward queues a copy of its
// status block into a pinned slot; the next forward (after its pair-count
// sync, which orders every earlier copy on that stream) or
// check_device_errors() reads them. Shared by all threads, because autograd
// runs backward on its own device thread.
struct ErrorRing {
  static constexpr int kSlots = 16;
  std::mutex mu;
  Tensor host;  // [kSlots, GSB_STATUS_WORDS] int32, pinned
  std::vector<at::cuda::CUDAEvent> events;
  std::array<cudaStream_t, kSlots> streams{};
  std::array<bool, kSlots> used{};
  int next = 0;

  void ensure() {
    if (!host.defined()) {
      host = at::empty({kSlots, GSB_STATUS_WORDS}, at::TensorOptions().dtype(at::kInt).pinned_memory(true));
      events.resize(kSlots);
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
    auto stream = at::cuda::getCurrentCUDAStream(status.device().index());
    host[i].copy_(status, /*non_blocking=*/true);
    events[i].record(stream);
    streams[i] = stream.stream();
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

// Pinned scalar for the pair total and the event that marks its copy.
struct PairRead {
  Tensor host;
  at::cuda::CUDAEvent done;
};
PairRead& pair_read() {
  thread_local PairRead* p = nullptr;
  if (p == nullptr) p = new PairRead();
  return *p;
}

// forward(means2d, conics, colors, opacities, depths [B,G,..] CUDA fp32, H, W,
//         alpha_thr, T_thr, bg[3], eps, max_alpha, save_state, pair_cap)
// pair_cap >= 0 raises the reference's overflow error when a tile holds more
// pairs than pair_cap (the overflow fallback disabled); -1 skips the check.
// Returns [out] (eval) or [out, perm, rec, tile_offsets, binned_ids, final_T,
// last_idx, pair_rec, status, render_ws] (training state).
std::vector<Tensor> forward(Tensor means2d, Tensor conics, Tensor colors, Tensor opacities, Tensor depths,
                            int64_t H, int64_t W, double alpha_thr, double T_thr, std::vector<double> bg,
                            double eps, double max_alpha, bool save_state, int64_t pair_cap) {
  const c10::cuda::CUDAGuard guard(means2d.device());
  const at::Device dev = means2d.device();
  const int64_t B = means2d.size(0), G = means2d.size(1), BG = B * G;
  gsb_raster_meta meta = make_meta(H, W, B, G, alpha_thr, T_thr, bg, eps, max_alpha);
  void* stream = stream_of(means2d);
  const Tensor m2 = aligned(means2d, 8);
  const Tensor q2 = conics.contiguous(), c2 = colors.contiguous(), o2 = opacities.contiguous(),
               d2 = depths.contiguous();

  const size_t ws_bytes = gsb_bin_prepare_workspace_size(&meta);
  Tensor status = empty({GSB_STATUS_WORDS}, at::kInt, dev);  // cleared by gsb_bin_count
  Tensor perm = empty({B, G}, at::kInt, dev);
  Tensor rec = empty({BG, GSB_REC_FLOATS}, at::kFloat, dev);
  Tensor pair_offsets = empty({BG + 1}, at::kInt, dev);
  Tensor tile_masks = empty({BG}, at::kLong, dev);
  Tensor ws = empty({static_cast<int64_t>(std::max<size_t>(ws_bytes, 1))}, at::kByte, dev);
  auto cur = at::cuda::getCurrentCUDAStream(dev.index());
  PairRead& pr = pair_read();
  {
    Phase ph("bin_prepare", means2d);
    check(gsb_bin_count(&meta, ptr<float>(m2), ptr<float>(q2), ptr<float>(o2), ptr<float>(d2), ptr<uint32_t>(status),
                        ws.data_ptr(), ws_bytes, stream),
          "gsb_bin_count");
    // The pair total is read as soon as the count kernel is done, while the
    // depth sort and scan run.
    if (!pr.host.defined()) pr.host = at::empty({1}, at::TensorOptions().dtype(at::kLong).pinned_memory(true));
    pr.host.copy_(status.narrow(0, GSB_STATUS_PAIR_TOTAL64, 2).view(at::kLong), /*non_blocking=*/true);
    pr.done.record(cur);
    check(gsb_bin_sort_scan(&meta, ptr<float>(m2), ptr<float>(q2), ptr<float>(c2), ptr<float>(o2), ptr<float>(d2),
                            ptr<int32_t>(perm), ptr<float>(rec), ptr<int32_t>(pair_offsets), ptr<uint64_t>(tile_masks),
                            ptr<uint32_t>(status),
                            ws.data_ptr(), ws_bytes, stream),
          "gsb_bin_sort_scan");
  }
  pr.done.synchronize();
  errors().check_all(cur.stream());  // every earlier copy on this stream is complete now
  const int64_t P = pr.host.data_ptr<int64_t>()[0];
  if (P >= (int64_t(1) << 31) - 1)
    throw std::runtime_error("gsplat_b200: " + std::to_string(P) + " tile-splat pairs exceed the supported 2^31 - 1");
  const int64_t T = B * ((H + 15) / 16) * ((W + 15) / 16);
  const size_t ws2_bytes = gsb_bin_emit_workspace_size(&meta, P);
  Tensor binned_ids = empty({P}, at::kInt, dev);
  Tensor tile_offsets = empty({T + 1}, at::kInt, dev);
  Tensor ws2 = empty({static_cast<int64_t>(std::max<size_t>(ws2_bytes, 1))}, at::kByte, dev);
  {
    Phase ph("bin_emit", means2d);
    check(gsb_bin_emit(&meta, ptr<float>(rec), ptr<int32_t>(pair_offsets), ptr<uint64_t>(tile_masks), P,
                       /*keys=*/nullptr,
                       ptr<int32_t>(binned_ids), ptr<int32_t>(tile_offsets), ptr<uint32_t>(status), ws2.data_ptr(),
                       ws2_bytes, stream),
          "gsb_bin_emit");
  }
  const bool dbg = debug_checks();
  if (dbg) read_status(status);
  if (pair_cap >= 0) {
    check(gsb_tile_stats(&meta, ptr<int32_t>(tile_offsets), ptr<uint32_t>(status), stream), "gsb_tile_stats");
    const auto v = read_status(status);
    if (static_cast<int64_t>(v[GSB_STATUS_MAX_TILE_COUNT]) > pair_cap)
      throw std::runtime_error("Tile overflow detected with max_fast_pairs=" + std::to_string(pair_cap) +
                               ". Enable overflow fallback or increase the runtime cap.");
  }

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
    Phase ph("render_fwd", means2d);
    check(gsb_render_forward(&meta, ptr<float>(rec), ptr<int32_t>(tile_offsets), ptr<int32_t>(binned_ids),
                             ptr<float>(out), ptr<float>(final_T), ptr<int32_t>(last_idx), ptr<float>(pair_rec),
                             ptr<uint32_t>(status), rws.data_ptr(), rws_bytes, stream),
          "gsb_render_forward");
  }
  if (dbg)
    read_status(status);
  else
    errors().defer(status);
  if (!save_state) return {out};
  return {out, perm, rec, tile_offsets, binned_ids, final_T, last_idx, pair_rec, status, rws};
}

// backward(perm, rec, tile_offsets, binned_ids, final_T, last_idx, pair_rec,
//          status, grad_out [B,H,W,3], H, W, alpha_thr, T_thr, bg, eps,
//          max_alpha, needs[4]) -> [g_means2d, g_conics, g_colors, g_opacities]
// (undefined where needs is false), in input order.
std::vector<Tensor> backward(Tensor perm, Tensor rec, Tensor tile_offsets, Tensor binned_ids, Tensor final_T,
                             Tensor last_idx, Tensor pair_rec, Tensor status, Tensor grad_out, int64_t H, int64_t W,
                             double alpha_thr, double T_thr, std::vector<double> bg, double eps, double max_alpha,
                             std::vector<bool> needs) {
  const c10::cuda::CUDAGuard guard(rec.device());
  const at::Device dev = rec.device();
  const int64_t B = perm.size(0), G = perm.size(1);
  gsb_raster_meta meta = make_meta(H, W, B, G, alpha_thr, T_thr, bg, eps, max_alpha);
  void* stream = stream_of(rec);
  const Tensor g = aligned(grad_out.to(at::kFloat), 16);
  const size_t ws_bytes = gsb_render_workspace_size(&meta);
  Tensor grad_rec = empty({B * G, GSB_REC_FLOATS}, at::kFloat, dev);
  Tensor ws = empty({static_cast<int64_t>(std::max<size_t>(ws_bytes, 1))}, at::kByte, dev);
  {
    Phase ph("render_bwd", rec);
    check(gsb_render_backward(&meta, ptr<float>(rec), ptr<int32_t>(tile_offsets), ptr<int32_t>(binned_ids),
                              ptr<float>(final_T), ptr<int32_t>(last_idx), ptr<float>(pair_rec), ptr<float>(g),
                              ptr<float>(grad_rec), ptr<uint32_t>(status), ws.data_ptr(), ws_bytes, stream),
          "gsb_render_backward");
  }
  Tensor gm, gc, gcol, go;
  if (needs.at(0)) gm = empty({B, G, 2}, at::kFloat, dev);
  if (needs.at(1)) gc = empty({B, G, 3}, at::kFloat, dev);
  if (needs.at(2)) gcol = empty({B, G, 3}, at::kFloat, dev);
  if (needs.at(3)) go = empty({B, G}, at::kFloat, dev);
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

PYBIND11_MODULE(_gsb_host, m) {
  m.doc() = "Native host runtime of the B200 rasterizer autograd path (drives the C ABI).";
  m.def("forward", &forward);
  m.def("backward", &backward);
  m.def("check_device_errors", &check_device_errors);
  m.def("set_phase_timing", &set_phase_timing);
  m.def("take_phase_times", &take_phase_times);
}
