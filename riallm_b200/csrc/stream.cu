// stream.cu -- layer streaming: a ring of device slots fed from pinned host
// memory on a side stream.
//
// riallm moves each layer's tensors to the device with synchronous copies
// from pageable memory on every forward (src/model.rs:1131-1201,
// src/memory.rs:113-125); its ModelOptions::prefetch_layers and
// prefetch_buffer_size (src/config.rs:389-393) are not acted on. Here a
// streamer owns `depth` device slots and a copy stream. prefetch(layer)
// copies the layer's packed bytes into slot layer % depth once the compute
// that last used that slot has released it (an event the copy stream waits
// on); acquire(layer) makes the compute stream wait for the copy's event;
// release(layer) records the compute stream's progress for the slot's next
// copy. No host synchronisation is involved, so copies of layers i+1 ..
// i+depth-1 overlap the compute of layer i.
//
// Copy timing uses a fixed ring of 4 x depth event pairs created with the
// streamer: a pair's elapsed time is added to the total when the pair is
// reused (waiting for that old copy if the host has run that far ahead of
// the copy stream) or when stats() is read, so a long streamed run keeps a
// constant number of events.
#include <vector>

#include "internal.h"

struct riallm_streamer {
  riallm_ctx* ctx = nullptr;
  int depth = 0;
  uint64_t slot_bytes = 0;
  char* dev = nullptr;
  bool owns_dev = false;
  cudaStream_t copy = nullptr;
  std::vector<cudaEvent_t> ready, freed;
  std::vector<int> layer;   // layer held by each slot, -1 when none
  std::vector<int> state;   // 0 empty, 1 copy issued, 2 acquired, 3 released
  std::vector<cudaEvent_t> t_start, t_stop;  // timing ring: one pair per copy in flight
  std::vector<char> t_pending;                // pair i timed a copy not yet added to copy_ms
  uint64_t bytes = 0, copies = 0;
  double copy_ms = 0.0;
};

namespace {

int fail(riallm_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

#define ST_CUDA(s, call, what)                                                        \
  do {                                                                                \
    cudaError_t e_ = (call);                                                          \
    if (e_ != cudaSuccess)                                                            \
      return fail((s)->ctx, RIALLM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// Adds the copy timed by ring pair i to the total (waiting for it to end).
int fold_timing(riallm_streamer* s, size_t i) {
  if (!s->t_pending[i]) return RIALLM_OK;
  ST_CUDA(s, cudaEventSynchronize(s->t_stop[i]), "cudaEventSynchronize");
  float ms = 0.f;
  ST_CUDA(s, cudaEventElapsedTime(&ms, s->t_start[i], s->t_stop[i]), "cudaEventElapsedTime");
  s->copy_ms += ms;
  s->t_pending[i] = 0;
  return RIALLM_OK;
}

void destroy(riallm_streamer* s) {
  if (!s) return;
  cudaSetDevice(s->ctx->device);
  if (s->copy) cudaStreamSynchronize(s->copy);
  for (auto e : s->ready) cudaEventDestroy(e);
  for (auto e : s->freed) cudaEventDestroy(e);
  for (auto e : s->t_start) cudaEventDestroy(e);
  for (auto e : s->t_stop) cudaEventDestroy(e);
  if (s->copy) cudaStreamDestroy(s->copy);
  if (s->owns_dev && s->dev) cudaFree(s->dev);
  delete s;
}

}  // namespace

extern "C" {

int32_t riallm_cuda_streamer_create(riallm_ctx* ctx, int32_t depth, uint64_t slot_bytes, void* device_slots,
                                    riallm_streamer** out) {
  if (!ctx || !out) return RIALLM_ERR_INVALID;
  *out = nullptr;
  if (depth < 1 || depth > 64 || slot_bytes == 0 || slot_bytes % 256 != 0)
    return fail(ctx, RIALLM_ERR_CONFIG, "streamer: depth must be 1..64 and slot_bytes a positive multiple of 256");
  if (device_slots && (reinterpret_cast<uintptr_t>(device_slots) & 255))
    return fail(ctx, RIALLM_ERR_INVALID, "streamer: device_slots must be 256-byte aligned");
  if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, RIALLM_ERR_CUDA, "cudaSetDevice");
  riallm_streamer* s = new riallm_streamer();
  s->ctx = ctx;
  s->depth = depth;
  s->slot_bytes = slot_bytes;
  s->layer.assign(depth, -1);
  s->state.assign(depth, 0);
  int rc = RIALLM_OK;
  if (device_slots) {
    s->dev = static_cast<char*>(device_slots);
  } else {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)slot_bytes * depth);
    if (e != cudaSuccess) rc = fail(ctx, RIALLM_ERR_MEMORY, std::string("streamer slots: ") + cudaGetErrorString(e));
    s->dev = static_cast<char*>(p);
    s->owns_dev = true;
  }
  if (rc == RIALLM_OK && cudaStreamCreateWithFlags(&s->copy, cudaStreamNonBlocking) != cudaSuccess)
    rc = fail(ctx, RIALLM_ERR_CUDA, "streamer: cudaStreamCreate");
  for (int i = 0; rc == RIALLM_OK && i < depth; ++i) {
    cudaEvent_t a, b;
    if (cudaEventCreateWithFlags(&a, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&b, cudaEventDisableTiming) != cudaSuccess) {
      rc = fail(ctx, RIALLM_ERR_CUDA, "streamer: cudaEventCreate");
      break;
    }
    s->ready.push_back(a);
    s->freed.push_back(b);
  }
  for (int i = 0; rc == RIALLM_OK && i < 4 * depth; ++i) {
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) {
      rc = fail(ctx, RIALLM_ERR_CUDA, "streamer: cudaEventCreate");
      break;
    }
    s->t_start.push_back(a);
    s->t_stop.push_back(b);
    s->t_pending.push_back(0);
  }
  if (rc != RIALLM_OK) {
    destroy(s);
    return rc;
  }
  *out = s;
  return RIALLM_OK;
}

int32_t riallm_cuda_streamer_destroy(riallm_streamer* s) {
  if (!s) return RIALLM_ERR_INVALID;
  destroy(s);
  return RIALLM_OK;
}

// Copies `n` byte ranges [offsets[i], offsets[i] + sizes[i]) of a layer's
// host blob to the same offsets of the layer's slot, after the slot's
// previous layer was released; one timing pair and one ready event for all.
static int32_t prefetch_ranges(riallm_streamer* s, int32_t layer, const char* host_src, const uint64_t* offsets,
                               const uint64_t* sizes, int32_t n) {
  uint64_t total = 0;
  for (int32_t i = 0; i < n; ++i) {
    if (offsets[i] > s->slot_bytes || sizes[i] > s->slot_bytes - offsets[i])
      return fail(s->ctx, RIALLM_ERR_MEMORY, "streamer: range [" + std::to_string(offsets[i]) + ", +" +
                                                 std::to_string(sizes[i]) + ") exceeds the slot size " +
                                                 std::to_string(s->slot_bytes));
    total += sizes[i];
  }
  const int slot = layer % s->depth;
  if (s->state[slot] == 1 || s->state[slot] == 2)
    return fail(s->ctx, RIALLM_ERR_CONFIG, "streamer: slot of layer " + std::to_string(layer) +
                                               " still holds unreleased layer " + std::to_string(s->layer[slot]));
  ST_CUDA(s, cudaSetDevice(s->ctx->device), "cudaSetDevice");
  // The slot's previous layer must be done with before it is overwritten.
  if (s->state[slot] == 3) ST_CUDA(s, cudaStreamWaitEvent(s->copy, s->freed[slot], 0), "wait slot release");
  const size_t ti = (size_t)(s->copies % s->t_start.size());
  if (int rc = fold_timing(s, ti)) return rc;
  cudaEvent_t a = s->t_start[ti], b = s->t_stop[ti];
  ST_CUDA(s, cudaEventRecord(a, s->copy), "cudaEventRecord");
  char* dst = s->dev + (uint64_t)slot * s->slot_bytes;
  for (int32_t i = 0; i < n; ++i)
    if (sizes[i])
      ST_CUDA(s, cudaMemcpyAsync(dst + offsets[i], host_src + offsets[i], sizes[i], cudaMemcpyHostToDevice, s->copy),
              "streamer H2D");
  ST_CUDA(s, cudaEventRecord(b, s->copy), "cudaEventRecord");
  s->t_pending[ti] = 1;
  ST_CUDA(s, cudaEventRecord(s->ready[slot], s->copy), "cudaEventRecord");
  s->layer[slot] = layer;
  s->state[slot] = 1;
  s->bytes += total;
  s->copies += 1;
  return RIALLM_OK;
}

int32_t riallm_cuda_streamer_prefetch(riallm_streamer* s, int32_t layer, const void* host_src, uint64_t bytes) {
  if (!s || !host_src || layer < 0) return RIALLM_ERR_INVALID;
  if (bytes > s->slot_bytes)
    return fail(s->ctx, RIALLM_ERR_MEMORY, "streamer: layer of " + std::to_string(bytes) +
                                               " bytes exceeds the slot size " + std::to_string(s->slot_bytes));
  const uint64_t off = 0;
  return prefetch_ranges(s, layer, static_cast<const char*>(host_src), &off, &bytes, 1);
}

int32_t riallm_cuda_streamer_prefetch_ranges(riallm_streamer* s, int32_t layer, const void* host_src,
                                             const uint64_t* offsets, const uint64_t* sizes, int32_t n) {
  if (!s || !host_src || layer < 0 || n < 0 || (n > 0 && (!offsets || !sizes))) return RIALLM_ERR_INVALID;
  return prefetch_ranges(s, layer, static_cast<const char*>(host_src), offsets, sizes, n);
}

int32_t riallm_cuda_streamer_acquire(riallm_streamer* s, int32_t layer, void* stream, void** dptr) {
  if (!s || !dptr || layer < 0) return RIALLM_ERR_INVALID;
  const int slot = layer % s->depth;
  if (s->layer[slot] != layer || s->state[slot] == 0 || s->state[slot] == 3)
    return fail(s->ctx, RIALLM_ERR_CONFIG, "streamer: layer " + std::to_string(layer) + " was not prefetched");
  ST_CUDA(s, cudaSetDevice(s->ctx->device), "cudaSetDevice");
  ST_CUDA(s, cudaStreamWaitEvent((cudaStream_t)stream, s->ready[slot], 0), "wait layer copy");
  s->state[slot] = 2;
  *dptr = s->dev + (uint64_t)slot * s->slot_bytes;
  return RIALLM_OK;
}

int32_t riallm_cuda_streamer_release(riallm_streamer* s, int32_t layer, void* stream) {
  if (!s || layer < 0) return RIALLM_ERR_INVALID;
  const int slot = layer % s->depth;
  if (s->layer[slot] != layer || s->state[slot] != 2)
    return fail(s->ctx, RIALLM_ERR_CONFIG, "streamer: layer " + std::to_string(layer) + " is not acquired");
  ST_CUDA(s, cudaSetDevice(s->ctx->device), "cudaSetDevice");
  ST_CUDA(s, cudaEventRecord(s->freed[slot], (cudaStream_t)stream), "cudaEventRecord");
  s->state[slot] = 3;
  return RIALLM_OK;
}

int32_t riallm_cuda_streamer_stats(riallm_streamer* s, uint64_t* bytes, uint64_t* copies, double* copy_ms) {
  if (!s) return RIALLM_ERR_INVALID;
  ST_CUDA(s, cudaSetDevice(s->ctx->device), "cudaSetDevice");
  ST_CUDA(s, cudaStreamSynchronize(s->copy), "cudaStreamSynchronize");
  for (size_t i = 0; i < s->t_start.size(); ++i)
    if (int rc = fold_timing(s, i)) return rc;
  if (bytes) *bytes = s->bytes;
  if (copies) *copies = s->copies;
  if (copy_ms) *copy_ms = s->copy_ms;
  return RIALLM_OK;
}

}  // extern "C"
