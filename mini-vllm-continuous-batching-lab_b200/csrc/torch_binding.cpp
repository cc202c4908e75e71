// Python binding of the per-step entry points (KV write, paged decode) that
// reads tensor metadata in C++ and calls the C ABI directly.
//
// The ctypes route marshals 20+ arguments per call and the Python wrapper
// queries each tensor attribute through the interpreter; together that is
// ~10-20 us of host time per call, more than the decode kernel itself at small
// batches.  Here one call costs about a microsecond on top of the launches.
//
// Only the common case is served: every argument check of the Python wrapper
// passes and no conversion is needed (contiguous last dimensions, int64 slot
// mapping and block table, int32 kv_len, all on the query's / key's device,
// 16-byte aligned query rows).  Anything else returns kSlowPath and the Python
// wrapper takes its full path, which performs the same conversions and raises
// the documented errors — so both routes give the same results and the same
// exceptions.
#include <torch/extension.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime_api.h>

#include <cmath>
#include <mutex>
#include <tuple>
#include <vector>

#include "mini_vllm_b200.h"

namespace {

constexpr int64_t kSlowPath = -1000;

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return MVB_DTYPE_BF16;
    case at::kHalf: return MVB_DTYPE_F16;
    case at::kFloat: return MVB_DTYPE_F32;
    default: return -1;
  }
}

// Decode workspaces owned by this binding, per device and per kernel family
// (the stream, split-K and scheduled kernels never share one), grown on demand
// and zero-filled when allocated.
std::mutex g_ws_mu;
std::vector<at::Tensor> g_ws[3];

// The stream and scheduled kernels' workspaces hold arrival counters (and the
// scheduled kernel's its schedule), so calls on different streams, which may
// overlap, each get their own.
struct StreamWorkspace {
  int dev;
  int kind;
  cudaStream_t stream;
  at::Tensor t;
};
std::vector<StreamWorkspace> g_ws_stream;

at::Tensor workspace(int dev, int kind, int64_t nbytes, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  auto zeros = [&]() { return at::zeros({nbytes}, at::TensorOptions().dtype(at::kByte).device(at::kCUDA, dev)); };
  if (kind == 0 || kind == 2) {
    for (StreamWorkspace& w : g_ws_stream) {
      if (w.dev != dev || w.kind != kind || w.stream != stream) continue;
      if (w.t.numel() < nbytes) w.t = zeros();
      return w.t;
    }
    g_ws_stream.push_back({dev, kind, stream, zeros()});
    return g_ws_stream.back().t;
  }
  std::vector<at::Tensor>& v = g_ws[kind];
  if ((int)v.size() <= dev) v.resize(dev + 1);
  at::Tensor& t = v[dev];
  if (!t.defined() || t.numel() < nbytes) t = zeros();
  return t;
}

// Duplicate-slot claim arrays owned by this binding, one per (device, pool
// slot count), each with the epoch of its last call (never 0; the array is
// cleared when the 32-bit epoch would wrap).
struct Claims {
  int dev;
  int64_t slots;
  at::Tensor arr;
  uint32_t epoch;
};
std::mutex g_claims_mu;
std::vector<Claims> g_claims;

std::pair<uint32_t*, uint32_t> next_claims(int dev, int64_t slots) {
  std::lock_guard<std::mutex> lock(g_claims_mu);
  for (Claims& c : g_claims) {
    if (c.dev != dev || c.slots != slots) continue;
    if (++c.epoch == 0xFFFFFFFFu) {
      c.arr.zero_();
      c.epoch = 1;
    }
    return {reinterpret_cast<uint32_t*>(c.arr.data_ptr<int32_t>()), c.epoch};
  }
  if (g_claims.size() >= 16) g_claims.erase(g_claims.begin());
  g_claims.push_back({dev, slots, at::zeros({slots}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev)), 1});
  return {reinterpret_cast<uint32_t*>(g_claims.back().arr.data_ptr<int32_t>()), 1};
}

int64_t kv_write(const at::Tensor& key, const at::Tensor& value, const at::Tensor& key_cache,
                 const at::Tensor& value_cache, const at::Tensor& slot_mapping, int64_t block_size,
                 bool check_duplicates, int64_t err_ptr) {
  if (!(key.dim() == 3 && key.sizes() == value.sizes() && key_cache.dim() == 4 &&
        key_cache.sizes() == value_cache.sizes() && slot_mapping.dim() == 1 &&
        slot_mapping.size(0) == key.size(0) && key.size(1) == key_cache.size(1) &&
        key.size(2) == key_cache.size(3) && block_size > 0 && block_size == key_cache.size(2) &&
        key.scalar_type() == key_cache.scalar_type() && value.scalar_type() == value_cache.scalar_type() &&
        dtype_code(key_cache.scalar_type()) >= 0 && key.is_cuda() &&
        key.get_device() == key_cache.get_device() && value.get_device() == value_cache.get_device() &&
        value_cache.get_device() == key_cache.get_device() && key_cache.is_contiguous() &&
        value_cache.is_contiguous() && key.stride(2) == 1 && value.stride(2) == 1 &&
        slot_mapping.scalar_type() == at::kLong && slot_mapping.get_device() == key.get_device() &&
        slot_mapping.is_contiguous()))
    return kSlowPath;
  const int64_t num_tokens = key.size(0);
  if (num_tokens == 0) return MVB_OK;
  const int dev = key.get_device();
  c10::cuda::CUDAGuard guard(dev);
  std::pair<uint32_t*, uint32_t> claims{nullptr, 0};
  if (check_duplicates) claims = next_claims(dev, key_cache.size(0) * block_size);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  return mvb_kv_cache_write(
      key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(), value.stride(0), value.stride(1),
      key_cache.data_ptr(), value_cache.data_ptr(), slot_mapping.data_ptr<int64_t>(), (int32_t)num_tokens,
      (int32_t)key.size(1), (int32_t)key.size(2), (int32_t)block_size, (int32_t)key_cache.size(0),
      dtype_code(key_cache.scalar_type()), claims.first, claims.second, reinterpret_cast<int32_t*>(err_ptr),
      stream);
}

std::tuple<int64_t, at::Tensor> decode(const at::Tensor& query, const at::Tensor& key_cache,
                                       const at::Tensor& value_cache, const at::Tensor& block_table,
                                       const at::Tensor& kv_len, int64_t block_size, double scale,
                                       const c10::optional<at::Tensor>& out_opt, int64_t variant,
                                       int64_t partition_tokens, int64_t err_ptr,
                                       const c10::optional<at::Tensor>& ws_opt) {
  const at::Tensor none;
  if (!(query.dim() == 3 && key_cache.dim() == 4 && key_cache.sizes() == value_cache.sizes() &&
        (query.size(2) == 64 || query.size(2) == 128) && block_size > 0 &&
        (block_size & (block_size - 1)) == 0 && key_cache.size(2) == block_size &&
        key_cache.size(3) == query.size(2) && key_cache.size(1) > 0 &&
        query.size(1) % key_cache.size(1) == 0 && dtype_code(query.scalar_type()) >= 0 &&
        key_cache.scalar_type() == query.scalar_type() && value_cache.scalar_type() == query.scalar_type() &&
        key_cache.is_contiguous() && value_cache.is_contiguous() && block_table.dim() == 2 &&
        block_table.size(0) == query.size(0) && kv_len.dim() == 1 && kv_len.size(0) == query.size(0) &&
        query.is_cuda() && key_cache.get_device() == query.get_device() &&
        value_cache.get_device() == query.get_device()))
    return {kSlowPath, none};
  const int dev = query.get_device();
  const int64_t esz = query.element_size();
  if (!(query.stride(2) == 1 && reinterpret_cast<uintptr_t>(query.data_ptr()) % 16 == 0 &&
        (query.stride(0) * esz) % 16 == 0 && (query.stride(1) * esz) % 16 == 0 &&
        block_table.scalar_type() == at::kLong && block_table.get_device() == dev && block_table.stride(1) == 1 &&
        kv_len.scalar_type() == at::kInt && kv_len.get_device() == dev && kv_len.is_contiguous()))
    return {kSlowPath, none};
  at::Tensor out;
  if (out_opt.has_value() && out_opt->defined()) {
    out = *out_opt;
    if (!(out.sizes() == query.sizes() && out.scalar_type() == query.scalar_type() &&
          out.get_device() == dev && out.stride(2) == 1))
      return {kSlowPath, none};
  } else {
    out = at::empty(query.sizes(), query.options());
  }
  const int64_t nd = query.size(0);
  if (nd == 0) return {MVB_OK, out};
  c10::cuda::CUDAGuard guard(dev);
  const int dt = dtype_code(query.scalar_type());
  int32_t v = 0, pt = 0, parts = 0;
  int64_t ws_bytes = 0;
  int st = mvb_paged_decode_plan(
      (int32_t)nd, (int32_t)query.size(1), (int32_t)key_cache.size(1), (int32_t)query.size(2),
      (int32_t)block_size, (int32_t)key_cache.size(0), (int32_t)block_table.size(1), dt, (int32_t)variant,
      (int32_t)partition_tokens, key_cache.data_ptr(), &v, &pt, &parts, &ws_bytes, nullptr);
  if (st != MVB_OK) return {st, out};
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  void* ws = nullptr;
  if (ws_opt.has_value() && ws_opt->defined()) {
    // the caller's workspace (a decode schedule built for this batch)
    const at::Tensor& w = *ws_opt;
    if (!(w.is_cuda() && w.get_device() == dev && w.numel() * w.element_size() >= ws_bytes))
      return {kSlowPath, none};
    ws = w.data_ptr();
    ws_bytes = w.numel() * w.element_size();
  } else if (ws_bytes > 0) {
    ws = workspace(dev, v == MVB_DECODE_STREAM ? 0 : v == MVB_DECODE_SCHED ? 2 : 1, ws_bytes, stream).data_ptr();
  }
  if (scale < 0) scale = std::pow((double)query.size(2), -0.5);  // the wrapper's default
  st = mvb_paged_decode(query.data_ptr(), query.stride(0), query.stride(1), key_cache.data_ptr(),
                        value_cache.data_ptr(), block_table.data_ptr<int64_t>(), block_table.stride(0),
                        (int32_t)block_table.size(1), kv_len.data_ptr<int32_t>(), out.data_ptr(), out.stride(0),
                        out.stride(1), (int32_t)nd, (int32_t)query.size(1), (int32_t)key_cache.size(1),
                        (int32_t)query.size(2), (int32_t)block_size, (int32_t)key_cache.size(0), (float)scale, dt,
                        (int32_t)variant, (int32_t)partition_tokens, ws, ws_bytes,
                        reinterpret_cast<int32_t*>(err_ptr), stream);
  return {st, out};
}

// Stream-ordered staging for a serving loop, one CUDA call each on raw handles
// (a torch.cuda.Stream's cuda_stream, a torch.cuda.Event's cuda_event): the
// torch-level copy_ / wait_event / record / set_stream calls cost about a
// microsecond of host time each, several per step.  Each returns the CUDA error
// code (0 = success).
// Wait (when wait_event != 0) for the event on `stream`, copy `nbytes` from
// `src` to `dst` (kind 0: host to device, 1: device to host), then record
// `record_event` (when != 0) on `stream`.
int64_t stream_copy(int64_t dst, int64_t src, int64_t nbytes, int64_t kind, int64_t stream, int64_t wait_event,
                    int64_t record_event) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  if (wait_event != 0) e = cudaStreamWaitEvent(s, reinterpret_cast<cudaEvent_t>(wait_event), 0);
  if (e == cudaSuccess && nbytes > 0)
    e = cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), (size_t)nbytes,
                        kind == 0 ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && record_event != 0) e = cudaEventRecord(reinterpret_cast<cudaEvent_t>(record_event), s);
  return (int64_t)e;
}

// `stream` waits for each of `events` (0 entries are skipped).
int64_t stream_wait_events(int64_t stream, const std::vector<int64_t>& events) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int64_t ev : events) {
    if (ev == 0) continue;
    const cudaError_t e = cudaStreamWaitEvent(s, reinterpret_cast<cudaEvent_t>(ev), 0);
    if (e != cudaSuccess) return (int64_t)e;
  }
  return 0;
}

int64_t event_record(int64_t event, int64_t stream) {
  return (int64_t)cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), reinterpret_cast<cudaStream_t>(stream));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "direct binding of the per-step C ABI calls (common case only; kSlowPath otherwise)";
  m.attr("SLOW_PATH") = kSlowPath;
  m.def("kv_write", &kv_write);
  m.def("decode", &decode);
  m.def("stream_copy", &stream_copy);
  m.def("stream_wait_events", &stream_wait_events);
  m.def("event_record", &event_record);
}
