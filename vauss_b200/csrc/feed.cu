// Dataset feed: packed RGBA8 ground truth staged ahead of the trainer.
//
// The reference's SceneLoader (crates/splat-train-dataset/src/scene_loader.rs:
// 59-184) runs loader actors that decode, pack (scene.rs:113-161) and hand
// batches through a 4-deep channel, keeping packed host copies in a byte-
// budgeted cache (:21-56).  Here decoded pixels are registered once; worker
// threads copy them into pinned host slots, the feed's copy stream moves them
// to device staging slots and one packing kernel writes the u32 words, all
// `ring_slots` batches ahead of the consumer.  The cache keeps packed views
// resident in HBM instead of host memory, so a cached visit copies nothing.
//
// Resources and their reuse rules (R = ring_slots, position p = the p-th
// batch of the sequence):
//   stage slot p % R   pinned host + device raw bytes; reused once the
//                      packing kernel of position p - R has finished (event);
//   output slot p % (R+H)  packed words of a streamed batch (H = batches the
//                      consumer holds at once); reused once the consumer's
//                      stream has passed the vs_feed_next call that hands out
//                      p + H (event recorded on the ctx stream);
//   ticket p % R       what position p became: output pointer, ready event.
// Position p is submitted by the vs_feed_next call that hands out p - R, after
// that call has recorded the release of p - R - H, the slot's last user, so
// every event a worker waits on was recorded before the job exists.
#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <chrono>
#include <cstring>
#include <deque>
#include <mutex>
#include <thread>
#include <vector>

#include "vs_internal.cuh"

namespace {

constexpr int kPackThreads = 256;
constexpr uint32_t kMaxSlots = 16;
constexpr auto kHostWaitLimit = std::chrono::seconds(60);

__device__ __forceinline__ uint32_t premul(uint32_t c, uint32_t a) { return (c * a + 127u) / 255u; }

__device__ __forceinline__ uint32_t pack_px(uint32_t r, uint32_t g, uint32_t b, uint32_t a, bool premultiply) {
  if (premultiply) {
    r = premul(r, a);
    g = premul(g, a);
    b = premul(b, a);
  }
  return r | (g << 8) | (b << 16) | (a << 24);
}

// Byte `i` of a little-endian word array.
__device__ __forceinline__ uint32_t byte_of(const uint32_t* w, int i) { return (w[i >> 2] >> ((i & 3) * 8)) & 0xffu; }

__device__ __forceinline__ uint32_t pack_from(const uint32_t* w, int px, int C, bool premultiply) {
  const int o = px * C;
  if (C == 1) {
    const uint32_t l = byte_of(w, o);
    return pack_px(l, l, l, 255u, false);
  }
  if (C == 2) {
    const uint32_t l = byte_of(w, o);
    return pack_px(l, l, l, byte_of(w, o + 1), premultiply);
  }
  if (C == 3) return pack_px(byte_of(w, o), byte_of(w, o + 1), byte_of(w, o + 2), 255u, false);
  return pack_px(byte_of(w, o), byte_of(w, o + 1), byte_of(w, o + 2), byte_of(w, o + 3), premultiply);
}

// Each thread packs 4 pixels: C 32-bit words in (16, 8 or 4-byte loads), one
// 16-byte store out.  HBM-bound; a grid-stride loop over groups.
template <int C>
__global__ void __launch_bounds__(kPackThreads) pack_kernel(const uint8_t* __restrict__ src, uint32_t pixels,
                                                             bool premultiply, uint32_t* __restrict__ out) {
  const uint32_t groups = pixels / 4;
  for (uint32_t q = blockIdx.x * blockDim.x + threadIdx.x; q < groups; q += gridDim.x * blockDim.x) {
    uint32_t w[C];
    if (C == 4) {
      const uint4 v = reinterpret_cast<const uint4*>(src)[q];
      w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
    } else if (C == 2) {
      const uint2 v = reinterpret_cast<const uint2*>(src)[q];
      w[0] = v.x, w[1] = v.y;
    } else {
      const uint32_t* s = reinterpret_cast<const uint32_t*>(src) + (size_t)q * C;
#pragma unroll
      for (int k = 0; k < C; ++k) w[k] = s[k];
    }
    uint4 o;
    o.x = pack_from(w, 0, C, premultiply);
    o.y = pack_from(w, 1, C, premultiply);
    o.z = pack_from(w, 2, C, premultiply);
    o.w = pack_from(w, 3, C, premultiply);
    reinterpret_cast<uint4*>(out)[q] = o;
  }
  // the last pixels / 4 remainder, one thread each, byte loads
  const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t px = groups * 4 + t;
  if (t < 4 && px < pixels) {
    const uint8_t* p = src + (size_t)px * C;
    uint32_t w[1] = {0};
    for (int k = 0; k < C; ++k) w[0] |= (uint32_t)p[k] << (8 * k);
    out[px] = pack_from(w, 0, C, premultiply);
  }
}

bool has_alpha_of(uint32_t channels) { return channels == 2 || channels == 4; }

cudaError_t launch_pack(cudaStream_t s, const uint8_t* src, uint32_t w, uint32_t h, uint32_t channels,
                        int32_t alpha_mode, uint32_t* out) {
  const uint32_t pixels = w * h;
  if (pixels == 0) return cudaSuccess;
  const bool pm = has_alpha_of(channels) && alpha_mode == VS_ALPHA_TRANSPARENT;
  const uint32_t blocks = std::max(1u, std::min(vs::div_up(vs::div_up(pixels, 4), kPackThreads), 148u * 16u));
  switch (channels) {
    case 1: pack_kernel<1><<<blocks, kPackThreads, 0, s>>>(src, pixels, pm, out); break;
    case 2: pack_kernel<2><<<blocks, kPackThreads, 0, s>>>(src, pixels, pm, out); break;
    case 3: pack_kernel<3><<<blocks, kPackThreads, 0, s>>>(src, pixels, pm, out); break;
    default: pack_kernel<4><<<blocks, kPackThreads, 0, s>>>(src, pixels, pm, out); break;
  }
  return cudaGetLastError();
}

// ---- the visiting order: epochs of seeded shuffles ----
uint64_t splitmix64(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Each epoch is a Fisher-Yates shuffle of all views, visited from the back
// (the reference's loaders shuffle and then pop, scene_loader.rs:131-136).
struct Sequencer {
  uint64_t state;
  uint32_t n;
  std::vector<uint32_t> epoch;
  Sequencer(uint64_t seed, uint32_t n_) : state(seed), n(n_) {}
  uint32_t next() {
    if (epoch.empty()) {
      epoch.resize(n);
      for (uint32_t i = 0; i < n; ++i) epoch[i] = i;
      for (uint32_t i = n - 1; i > 0; --i) {
        const uint32_t j = (uint32_t)(((unsigned __int128)splitmix64(state) * (uint64_t)(i + 1)) >> 64);
        std::swap(epoch[i], epoch[j]);
      }
    }
    const uint32_t v = epoch.back();
    epoch.pop_back();
    return v;
  }
};

struct FeedView {
  const uint8_t* px = nullptr;
  uint32_t w = 0, h = 0, c = 0;
  int32_t alpha_mode = 0;
  bool set = false;
  uint32_t* resident = nullptr;  // packed copy kept in HBM (admitted to the cache)
  cudaEvent_t ready = nullptr;   // recorded after the resident copy is packed
  bool ready_recorded = false;
  size_t raw_bytes() const { return (size_t)w * h * c; }
  size_t packed_bytes() const { return (size_t)w * h * 4; }
};

struct Ticket {
  uint64_t pos = ~0ull;
  uint32_t view = 0;
  uint32_t* out = nullptr;
  int out_slot = -1;           // -1: resident
  bool cached = false;
  bool issued = false;
  uint64_t h2d = 0;
  cudaEvent_t ready = nullptr;
  vs_status st = VS_OK;
  std::string msg;
};

struct Job {
  uint64_t pos;
  uint32_t view;
  uint32_t* out;
  int out_slot;
  bool admit;         // pack into the view's resident buffer
  bool wait_release;  // the output slot was handed out before: wait for its release
  bool slot_used;     // the stage slot was used before: wait for its last packing
};

}  // namespace

struct vs_feed {
  vs_ctx* ctx = nullptr;
  int device = 0;
  vs_feed_cfg cfg{};
  std::vector<FeedView> views;
  Sequencer seq{0, 0};
  bool started = false;
  vs_status failed = VS_OK;  // a start that failed part-way leaves the feed unusable
  std::string failed_msg;
  uint64_t next_pos = 0;     // next position to hand out
  std::deque<int> held;      // output slots of the batches the consumer holds (-1: resident)
  uint64_t cache_used = 0;
  cudaStream_t copy = nullptr;
  size_t slot_raw = 0, slot_px = 0;
  std::vector<uint8_t*> host_stage, dev_stage;
  std::vector<cudaEvent_t> stage_done;
  std::vector<char> stage_used;  // written and read under mu
  std::vector<uint32_t*> out_slots;
  std::vector<cudaEvent_t> out_released;
  std::vector<char> out_ever_released;  // written and read under mu
  std::vector<Ticket> tickets;
  std::mutex mu;                 // queue, tickets, views' cache state
  std::condition_variable cv_job, cv_done;
  std::mutex issue_mu;           // keeps one job's stream operations together
  std::deque<Job> queue;
  std::vector<std::thread> workers;
  bool stop = false;
  std::atomic<uint64_t> launches{0};
};

namespace {

void worker_main(vs_feed* f) {
  cudaSetDevice(f->device);
  const uint32_t R = f->cfg.ring_slots;
  for (;;) {
    Job job;
    {
      std::unique_lock<std::mutex> lk(f->mu);
      f->cv_job.wait(lk, [&] { return f->stop || !f->queue.empty(); });
      if (f->stop) return;
      job = f->queue.front();
      f->queue.pop_front();
      job.slot_used = f->stage_used[job.pos % R] != 0;
    }
    const uint32_t s = (uint32_t)(job.pos % R);
    const FeedView& v = f->views[job.view];
    const size_t raw = v.raw_bytes();
    cudaError_t e = cudaSuccess;
    const char* what = "";
    // the previous user of this stage slot (position pos - R) was issued
    // before this job was submitted; wait for its copy and packing to end
    if (job.slot_used) {
      e = cudaEventSynchronize(f->stage_done[s]);
      what = "feed: stage slot wait";
    }
    if (e == cudaSuccess) std::memcpy(f->host_stage[s], v.px, raw);
    if (e == cudaSuccess) {
      std::lock_guard<std::mutex> ik(f->issue_mu);
      if (job.wait_release) {
        e = cudaStreamWaitEvent(f->copy, f->out_released[job.out_slot], 0);
        what = "feed: wait for output slot";
      }
      if (e == cudaSuccess) {
        e = cudaMemcpyAsync(f->dev_stage[s], f->host_stage[s], raw, cudaMemcpyHostToDevice, f->copy);
        what = "feed: host-to-device copy";
      }
      if (e == cudaSuccess) {
        e = launch_pack(f->copy, f->dev_stage[s], v.w, v.h, v.c, v.alpha_mode, job.out);
        what = "feed: packing kernel";
        f->launches += (v.w * v.h) ? 1 : 0;
      }
      if (e == cudaSuccess) e = cudaEventRecord(f->stage_done[s], f->copy);
      Ticket& t = f->tickets[job.pos % R];
      if (e == cudaSuccess) e = cudaEventRecord(t.ready, f->copy);
      if (e == cudaSuccess && job.admit) e = cudaEventRecord(f->views[job.view].ready, f->copy);
    }
    {
      std::lock_guard<std::mutex> lk(f->mu);
      f->stage_used[s] = 1;
      Ticket& t = f->tickets[job.pos % R];
      t.h2d = raw;
      if (e != cudaSuccess) {
        t.st = VS_ERR_CUDA;
        t.msg = std::string(what) + ": " + cudaGetErrorString(e);
      }
      if (job.admit && e == cudaSuccess) f->views[job.view].ready_recorded = true;
      t.issued = true;
    }
    f->cv_done.notify_all();
  }
}

// Decides what position `pos` becomes and queues its staging job (if any).
// Called by the consumer thread with f->mu held.
vs_status submit(vs_feed* f, uint64_t pos) {
  const uint32_t R = f->cfg.ring_slots;
  const uint32_t v = f->seq.next();
  FeedView& view = f->views[v];
  Ticket& t = f->tickets[pos % R];
  t.pos = pos;
  t.view = v;
  t.st = VS_OK;
  t.msg.clear();
  t.h2d = 0;
  if (view.resident) {  // a cache hit: nothing to copy
    t.out = view.resident;
    t.out_slot = -1;
    t.cached = true;
    t.issued = true;
    return VS_OK;
  }
  bool admit = false;
  if (f->cfg.cache_bytes > 0 && f->cache_used + view.packed_bytes() < f->cfg.cache_bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, std::max<size_t>(view.packed_bytes(), 16)) == cudaSuccess) {
      view.resident = static_cast<uint32_t*>(p);
      f->cache_used += view.packed_bytes();
      admit = true;
    } else {
      cudaGetLastError();  // out of HBM: stream this view instead
    }
  }
  t.cached = admit;
  t.issued = false;
  t.out_slot = admit ? -1 : (int)(pos % (R + f->cfg.hold));
  t.out = admit ? view.resident : f->out_slots[t.out_slot];
  const bool wait_release = t.out_slot >= 0 && f->out_ever_released[t.out_slot] != 0;
  f->queue.push_back(Job{pos, v, t.out, t.out_slot, admit, wait_release, false});
  f->cv_job.notify_one();
  return VS_OK;
}

vs_status start(vs_feed* f) {
  vs_ctx* ctx = f->ctx;
  const uint32_t R = f->cfg.ring_slots;
  for (uint32_t i = 0; i < f->cfg.num_views; ++i) {
    const FeedView& v = f->views[i];
    if (!v.set) return vs_fail(ctx, VS_ERR_INVALID, "feed: view %u was never set", i);
    f->slot_raw = std::max(f->slot_raw, v.raw_bytes());
    f->slot_px = std::max(f->slot_px, (size_t)v.w * v.h);
  }
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  VS_CUDA(ctx, cudaStreamCreateWithFlags(&f->copy, cudaStreamNonBlocking));
  const size_t raw = std::max<size_t>(f->slot_raw, 16), px = std::max<size_t>(f->slot_px, 4);
  f->host_stage.assign(R, nullptr);
  f->dev_stage.assign(R, nullptr);
  f->stage_done.assign(R, nullptr);
  f->stage_used.assign(R, 0);
  for (uint32_t s = 0; s < R; ++s) {
    VS_CUDA(ctx, cudaHostAlloc(reinterpret_cast<void**>(&f->host_stage[s]), raw, cudaHostAllocDefault));
    VS_CUDA(ctx, cudaMalloc(reinterpret_cast<void**>(&f->dev_stage[s]), raw));
    // the workers wait on these from the host: a blocking-sync event puts the
    // waiting thread to sleep instead of spinning a core, which one process
    // per GPU with several workers each would oversubscribe
    VS_CUDA(ctx, cudaEventCreateWithFlags(&f->stage_done[s], cudaEventDisableTiming | cudaEventBlockingSync));
  }
  const uint32_t outs = R + f->cfg.hold;
  f->out_slots.assign(outs, nullptr);
  f->out_released.assign(outs, nullptr);
  f->out_ever_released.assign(outs, 0);
  for (uint32_t s = 0; s < outs; ++s) {
    VS_CUDA(ctx, cudaMalloc(reinterpret_cast<void**>(&f->out_slots[s]), px * 4));
    VS_CUDA(ctx, cudaEventCreateWithFlags(&f->out_released[s], cudaEventDisableTiming));
  }
  f->tickets.resize(R);
  for (uint32_t s = 0; s < R; ++s) VS_CUDA(ctx, cudaEventCreateWithFlags(&f->tickets[s].ready, cudaEventDisableTiming));
  for (auto& v : f->views) VS_CUDA(ctx, cudaEventCreateWithFlags(&v.ready, cudaEventDisableTiming));
  const uint32_t nw = f->cfg.workers ? std::min(f->cfg.workers, kMaxSlots) : R;
  for (uint32_t i = 0; i < nw; ++i) f->workers.emplace_back(worker_main, f);
  f->started = true;
  std::lock_guard<std::mutex> lk(f->mu);
  for (uint32_t p = 0; p < R; ++p) VS_TRY(submit(f, p));
  return VS_OK;
}

}  // namespace

VS_API vs_status vs_pack_view(vs_ctx* ctx, const uint8_t* pixels, uint32_t width, uint32_t height,
                              uint32_t channels, int32_t alpha_mode, uint32_t* out, int32_t* has_alpha) {
  if (!ctx) return VS_ERR_INVALID;
  if (channels < 1 || channels > 4) return vs_fail(ctx, VS_ERR_INVALID, "pack_view: %u channels", channels);
  if (alpha_mode != VS_ALPHA_MASKED && alpha_mode != VS_ALPHA_TRANSPARENT)
    return vs_fail(ctx, VS_ERR_INVALID, "pack_view: alpha mode %d", alpha_mode);
  if ((uint64_t)width * height >= (1ull << 31)) return vs_fail(ctx, VS_ERR_CAPACITY, "pack_view: %ux%u", width, height);
  if (has_alpha) *has_alpha = has_alpha_of(channels) ? 1 : 0;
  if ((uint64_t)width * height == 0) return VS_OK;
  if (!pixels || !out) return vs_fail(ctx, VS_ERR_INVALID, "pack_view: null argument");
  if ((reinterpret_cast<uintptr_t>(pixels) | reinterpret_cast<uintptr_t>(out)) & 15)
    return vs_fail(ctx, VS_ERR_INVALID, "pack_view: pixels and out must be 16-byte aligned");
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  ++ctx->launches;
  return vs_cuda(ctx, launch_pack(ctx->stream, pixels, width, height, channels, alpha_mode, out), "pack_view launch");
}

VS_API vs_status vs_feed_create(vs_ctx* ctx, const vs_feed_cfg* cfg, vs_feed** out) {
  if (!ctx) return VS_ERR_INVALID;
  if (!cfg || !out) return vs_fail(ctx, VS_ERR_INVALID, "feed_create: null argument");
  *out = nullptr;
  if (cfg->num_views == 0) return vs_fail(ctx, VS_ERR_INVALID, "feed_create: no views");
  if (cfg->ring_slots < 2 || cfg->ring_slots > kMaxSlots)
    return vs_fail(ctx, VS_ERR_INVALID, "feed_create: ring_slots %u (2..%u)", cfg->ring_slots, kMaxSlots);
  if (cfg->hold < 1 || cfg->hold > kMaxSlots)
    return vs_fail(ctx, VS_ERR_INVALID, "feed_create: hold %u (1..%u)", cfg->hold, kMaxSlots);
  vs_feed* f = new vs_feed();
  f->ctx = ctx;
  f->device = ctx->device;
  f->cfg = *cfg;
  f->views.resize(cfg->num_views);
  f->seq = Sequencer(cfg->seed, cfg->num_views);
  *out = f;
  return VS_OK;
}

VS_API vs_status vs_feed_set_view(vs_feed* f, uint32_t index, const uint8_t* pixels, uint32_t width, uint32_t height,
                                  uint32_t channels, int32_t alpha_mode) {
  if (!f) return VS_ERR_INVALID;
  vs_ctx* ctx = f->ctx;
  if (f->started) return vs_fail(ctx, VS_ERR_INVALID, "feed_set_view: the feed has started");
  if (index >= f->cfg.num_views) return vs_fail(ctx, VS_ERR_INVALID, "feed_set_view: view %u of %u", index, f->cfg.num_views);
  if (channels < 1 || channels > 4) return vs_fail(ctx, VS_ERR_INVALID, "feed_set_view: %u channels", channels);
  if (alpha_mode != VS_ALPHA_MASKED && alpha_mode != VS_ALPHA_TRANSPARENT)
    return vs_fail(ctx, VS_ERR_INVALID, "feed_set_view: alpha mode %d", alpha_mode);
  if ((uint64_t)width * height == 0 || (uint64_t)width * height >= (1ull << 31))
    return vs_fail(ctx, VS_ERR_INVALID, "feed_set_view: image size %ux%u", width, height);
  if (!pixels) return vs_fail(ctx, VS_ERR_INVALID, "feed_set_view: null pixels");
  FeedView& v = f->views[index];
  v.px = pixels;
  v.w = width, v.h = height, v.c = channels;
  v.alpha_mode = alpha_mode;
  v.set = true;
  return VS_OK;
}

VS_API vs_status vs_feed_next(vs_feed* f, vs_scene_batch* out) {
  if (!f) return VS_ERR_INVALID;
  vs_ctx* ctx = f->ctx;
  if (!out) return vs_fail(ctx, VS_ERR_INVALID, "feed_next: null batch");
  if (f->failed != VS_OK) return vs_fail(ctx, f->failed, "feed_next: the feed failed to start: %s", f->failed_msg.c_str());
  if (!f->started) {
    const vs_status st = start(f);
    if (st != VS_OK) {
      f->failed = st;
      f->failed_msg = ctx->err;
      return st;
    }
  }
  VS_CUDA(ctx, cudaSetDevice(ctx->device));
  const uint32_t R = f->cfg.ring_slots;
  // the consumer is done with batch pos - hold once its stream passes here
  if (f->held.size() >= f->cfg.hold) {
    const int o = f->held.front();
    f->held.pop_front();
    if (o >= 0) {
      VS_CUDA(ctx, cudaEventRecord(f->out_released[o], ctx->stream));
      std::lock_guard<std::mutex> lk(f->mu);
      f->out_ever_released[o] = 1;
    }
  }
  const uint64_t pos = f->next_pos;
  Ticket* t = &f->tickets[pos % R];
  std::unique_lock<std::mutex> lk(f->mu);
  bool ok = f->cv_done.wait_for(lk, kHostWaitLimit, [&] {
    if (!t->issued) return false;
    // a hit on a view whose resident copy is still being staged waits for it
    return !t->cached || t->st != VS_OK || f->views[t->view].ready_recorded;
  });
  if (!ok) return vs_fail(ctx, VS_ERR_DEVICE_TIMEOUT, "feed_next: staging of batch %llu did not finish in 60 s",
                          (unsigned long long)pos);
  if (t->st != VS_OK) return vs_fail(ctx, t->st, "%s", t->msg.c_str());
  const FeedView& v = f->views[t->view];
  cudaEvent_t ready = t->cached ? v.ready : t->ready;
  VS_CUDA(ctx, cudaStreamWaitEvent(ctx->stream, ready, 0));
  out->img_packed = t->out;
  out->width = v.w;
  out->height = v.h;
  out->view_index = t->view;
  out->has_alpha = has_alpha_of(v.c) ? 1 : 0;
  out->alpha_mode = v.alpha_mode;
  out->cached = t->cached ? 1 : 0;
  out->h2d_bytes = t->h2d;
  f->held.push_back(t->out_slot);
  f->next_pos = pos + 1;
  VS_TRY(submit(f, pos + R));
  lk.unlock();
  ctx->launches += f->launches.exchange(0);
  return VS_OK;
}

VS_API void vs_feed_destroy(vs_feed* f) {
  if (!f) return;
  {
    std::lock_guard<std::mutex> lk(f->mu);
    f->stop = true;
  }
  f->cv_job.notify_all();
  for (auto& w : f->workers) w.join();
  // does not touch f->ctx, which may be gone already; cudaFree below waits
  // for the device, so no consumer still reads a slot that is freed
  cudaSetDevice(f->device);
  if (f->copy) cudaStreamSynchronize(f->copy);
  for (auto p : f->host_stage) if (p) cudaFreeHost(p);
  for (auto p : f->dev_stage) if (p) cudaFree(p);
  for (auto p : f->out_slots) if (p) cudaFree(p);
  for (auto e : f->stage_done) if (e) cudaEventDestroy(e);
  for (auto e : f->out_released) if (e) cudaEventDestroy(e);
  for (auto& t : f->tickets) if (t.ready) cudaEventDestroy(t.ready);
  for (auto& v : f->views) {
    if (v.resident) cudaFree(v.resident);
    if (v.ready) cudaEventDestroy(v.ready);
  }
  if (f->copy) cudaStreamDestroy(f->copy);
  delete f;
}

VS_API vs_status vs_feed_order(uint64_t seed, uint32_t num_views, uint32_t count, uint32_t* out) {
  if (num_views == 0 || (count && !out)) return VS_ERR_INVALID;
  Sequencer s(seed, num_views);
  for (uint32_t i = 0; i < count; ++i) out[i] = s.next();
  return VS_OK;
}
