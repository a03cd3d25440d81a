// Stable LSD radix sort of (u32 key, u32 value) pairs and a device-wide
// inclusive scan.
//
// Replaces the reference's radix_argsort_with_count
// (crates/splat-train-sort/src/lib.rs:40-189, kernels.rs:13-341: 8-bit digits,
// count / reduce / scan / scan_add / scatter per pass) and prefix sums
// (crates/splat-train-scan/src/kernels.rs:30-212).
//
// Per pass of an 8- or 9-bit digit: (1) each block histograms its 2048-key
// tile into a digit-major table hist[digit][tile]; (2) an exclusive scan of
// that table gives every (digit, tile) its global output offset; (3) each
// block ranks its keys stably (every warp ranks a contiguous 256-key slice,
// equal digits found by one ballot per digit bit, warps are combined through
// per-digit counts), scatters them into shared memory in digit order and
// writes contiguous per-digit runs to global memory.  A sort of b key bits
// takes ceil(b / 9) passes, the bits split as evenly as possible over them; a
// stable LSD sort gives the same order whatever the digit widths.
#include <cuda/atomic>
#include <mutex>

#include "vs_internal.cuh"

namespace {

using namespace vs;

constexpr uint32_t SORT_THREADS = 256;
constexpr uint32_t SORT_WARPS = SORT_THREADS / 32;
constexpr uint32_t ITEMS = 8;  // per thread
constexpr uint32_t SORT_TILE = SORT_THREADS * ITEMS;  // 2048
constexpr uint32_t RADIX = 256;       // 8-bit digits: the table size of the fixed-scratch sort
constexpr uint32_t MAX_DIGIT_BITS = 9;

template <uint32_t RB>
__global__ void __launch_bounds__(SORT_THREADS) hist_kernel(const uint32_t* __restrict__ keys, uint32_t count,
                                                            uint32_t shift, uint32_t mask, uint32_t tiles,
                                                            uint32_t* __restrict__ hist, uint32_t sub = 0u) {
  constexpr uint32_t R = 1u << RB;
  __shared__ uint32_t s_hist[R];
  const uint32_t tid = threadIdx.x;
  for (uint32_t d = tid; d < R; d += SORT_THREADS) s_hist[d] = 0;
  __syncthreads();
  const uint32_t base = blockIdx.x * SORT_TILE;
#pragma unroll
  for (uint32_t r = 0; r < ITEMS; ++r) {
    const uint32_t i = base + r * SORT_THREADS + tid;
    const bool valid = i < count;
    // plain shared-memory atomics: cheaper on sm_100 than grouping equal
    // digits with match_any first
    if (valid) atomicAdd(&s_hist[((keys[i] - sub) >> shift) & mask], 1u);
  }
  __syncthreads();
  // the table holds the pass's mask + 1 digits only
  for (uint32_t d = tid; d <= mask; d += SORT_THREADS) hist[d * tiles + blockIdx.x] = s_hist[d];
}

template <uint32_t RB>
__global__ void __launch_bounds__(SORT_THREADS) scatter_kernel(
    const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in, uint32_t* __restrict__ keys_out,
    uint32_t* __restrict__ vals_out, uint32_t count, uint32_t shift, uint32_t mask, uint32_t tiles,
    const uint32_t* __restrict__ offsets /* exclusive-scanned hist, digit-major */,
    // optional: keys_in - sub are the keys; vals_in NULL gives the values
    // 0..count-1; with gout, gout[out] = gsrc[value] beside every output
    uint32_t sub = 0u, const uint32_t* __restrict__ gsrc = nullptr, uint32_t* __restrict__ gout = nullptr) {
  constexpr uint32_t R = 1u << RB;
  constexpr uint32_t DPT = R / SORT_THREADS;  // digits per thread, consecutive
  static_assert(DPT >= 1 && DPT * SORT_THREADS == R, "digit ownership");
  __shared__ uint32_t s_wcnt[SORT_WARPS][R];  // per-warp digit counts, then per-warp offsets
  __shared__ uint32_t s_dstart[R];            // block-local start of each digit
  __shared__ uint32_t s_goff[R];              // global start of each digit for this tile
  __shared__ uint32_t s_keys[SORT_TILE];
  __shared__ uint32_t s_vals[SORT_TILE];
  __shared__ uint32_t s_scan[SORT_WARPS];
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  for (uint32_t i = tid; i < SORT_WARPS * R; i += SORT_THREADS) (&s_wcnt[0][0])[i] = 0;
#pragma unroll
  for (uint32_t j = 0; j < DPT; ++j) {
    const uint32_t dg = tid * DPT + j;
    if (dg <= mask) s_goff[dg] = offsets[dg * tiles + blockIdx.x];  // no key holds a larger digit
  }
  __syncthreads();

  // Warp `warp` owns keys [base + warp*256, base + warp*256 + 256), 32 per round.
  const uint32_t base = blockIdx.x * SORT_TILE + warp * (ITEMS * 32);
  uint32_t k[ITEMS], v[ITEMS], d[ITEMS], rank[ITEMS];
#pragma unroll
  for (uint32_t r = 0; r < ITEMS; ++r) {
    const uint32_t i = base + r * 32 + lane;
    const bool valid = i < count;
    k[r] = valid ? keys_in[i] - sub : 0u;
    v[r] = valid ? (vals_in ? vals_in[i] : i) : 0u;
    d[r] = valid ? ((k[r] >> shift) & mask) : R;
  }
#pragma unroll
  for (uint32_t r = 0; r < ITEMS; ++r) {
    // lanes holding the same digit (RB + 1 bits: an invalid lane holds R), by
    // one ballot per bit -- cheaper on sm_100 than match_any
    uint32_t peers = 0xffffffffu;
#pragma unroll
    for (uint32_t b = 0; b <= RB; ++b) {
      const uint32_t bit = (d[r] >> b) & 1u;
      const uint32_t bal = __ballot_sync(0xffffffffu, bit);
      peers &= bit ? bal : ~bal;
    }
    const uint32_t leader = __ffs(peers) - 1;
    uint32_t before = 0;
    if (lane == leader && d[r] < R) {
      before = s_wcnt[warp][d[r]];
      s_wcnt[warp][d[r]] = before + __popc(peers);
    }
    before = __shfl_sync(0xffffffffu, before, leader);
    rank[r] = before + __popc(peers & ((1u << lane) - 1u));
    __syncwarp();
  }
  __syncthreads();
  // thread `tid` owns digits tid*DPT .. tid*DPT + DPT-1: exclusive prefix over
  // warps, block totals
  uint32_t dtot[DPT];
  uint32_t run = 0;
#pragma unroll
  for (uint32_t j = 0; j < DPT; ++j) {
    const uint32_t dg = tid * DPT + j;
    uint32_t acc = 0;
#pragma unroll
    for (uint32_t w = 0; w < SORT_WARPS; ++w) {
      const uint32_t c = s_wcnt[w][dg];
      s_wcnt[w][dg] = acc;
      acc += c;
    }
    dtot[j] = acc;
    run += acc;
  }
  // exclusive scan of the digit totals across the block (digit-ordered)
  uint32_t incl = run;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= (uint32_t)off) incl += y;
  }
  if (lane == 31) s_scan[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t s = lane < SORT_WARPS ? s_scan[lane] : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= (uint32_t)off) s += y;
    }
    if (lane < SORT_WARPS) s_scan[lane] = s;
  }
  __syncthreads();
  uint32_t start = incl - run + (warp ? s_scan[warp - 1] : 0u);
#pragma unroll
  for (uint32_t j = 0; j < DPT; ++j) {
    s_dstart[tid * DPT + j] = start;
    start += dtot[j];
  }
  __syncthreads();
#pragma unroll
  for (uint32_t r = 0; r < ITEMS; ++r) {
    if (d[r] < R) {
      const uint32_t pos = s_dstart[d[r]] + s_wcnt[warp][d[r]] + rank[r];
      s_keys[pos] = k[r];
      s_vals[pos] = v[r];
    }
  }
  __syncthreads();
  const uint32_t tile_base = blockIdx.x * SORT_TILE;
  const uint32_t n_here = min(SORT_TILE, count - tile_base);
  for (uint32_t p = tid; p < n_here; p += SORT_THREADS) {
    const uint32_t key = s_keys[p];
    const uint32_t dd = (key >> shift) & mask;
    const uint32_t out = s_goff[dd] + (p - s_dstart[dd]);
    keys_out[out] = key;
    const uint32_t val = s_vals[p];
    vals_out[out] = val;
    if (gout) gout[out] = gsrc[val];
  }
}

// ---- device-wide inclusive scan of u32 (three phases) ----
constexpr uint32_t SCAN_THREADS = 256;
constexpr uint32_t SCAN_ITEMS = 16;
constexpr uint32_t SCAN_CHUNK = SCAN_THREADS * SCAN_ITEMS;  // 4096

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t x, uint32_t* s_warp, uint32_t* total) {
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  uint32_t incl = x;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= (uint32_t)off) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t s = lane < (blockDim.x >> 5) ? s_warp[lane] : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= (uint32_t)off) s += y;
    }
    s_warp[lane] = s;
  }
  __syncthreads();
  const uint32_t res = incl - x + (warp ? s_warp[warp - 1] : 0u);
  *total = s_warp[(blockDim.x >> 5) - 1];
  __syncthreads();
  return res;
}

__global__ void __launch_bounds__(SCAN_THREADS) scan_reduce_kernel(const uint32_t* __restrict__ data, uint32_t count,
                                                                   uint32_t* __restrict__ sums) {
  __shared__ uint32_t s_warp[32];
  const uint32_t base = blockIdx.x * SCAN_CHUNK + threadIdx.x * SCAN_ITEMS;
  uint32_t s = 0;
#pragma unroll
  for (uint32_t i = 0; i < SCAN_ITEMS; ++i) s += (base + i < count) ? data[base + i] : 0u;
  uint32_t total;
  block_exclusive_scan(s, s_warp, &total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// One block: exclusive scan of the chunk sums in place; total to *total_dev.
__global__ void __launch_bounds__(1024) scan_sums_kernel(uint32_t* sums, uint32_t nsums,
                                                         unsigned long long* total_dev) {
  __shared__ uint32_t s_warp[32];
  const uint32_t per = (nsums + blockDim.x - 1) / blockDim.x;
  const uint32_t b0 = threadIdx.x * per;
  uint32_t local = 0;
  for (uint32_t i = 0; i < per; ++i) local += (b0 + i < nsums) ? sums[b0 + i] : 0u;
  uint32_t total;
  uint32_t run = block_exclusive_scan(local, s_warp, &total);
  for (uint32_t i = 0; i < per; ++i) {
    if (b0 + i < nsums) {
      const uint32_t x = sums[b0 + i];
      sums[b0 + i] = run;
      run += x;
    }
  }
  if (threadIdx.x == 0 && total_dev) *total_dev = total;
}

template <bool kInclusive>
__global__ void __launch_bounds__(SCAN_THREADS) scan_apply_kernel(uint32_t* __restrict__ data, uint32_t count,
                                                                  const uint32_t* __restrict__ sums) {
  __shared__ uint32_t s_warp[32];
  const uint32_t base = blockIdx.x * SCAN_CHUNK + threadIdx.x * SCAN_ITEMS;
  uint32_t x[SCAN_ITEMS];
  uint32_t s = 0;
#pragma unroll
  for (uint32_t i = 0; i < SCAN_ITEMS; ++i) {
    x[i] = (base + i < count) ? data[base + i] : 0u;
    s += x[i];
  }
  uint32_t total;
  uint32_t run = block_exclusive_scan(s, s_warp, &total) + sums[blockIdx.x];
#pragma unroll
  for (uint32_t i = 0; i < SCAN_ITEMS; ++i) {
    if (kInclusive) run += x[i];
    if (base + i < count) data[base + i] = run;
    if (!kInclusive) run += x[i];
  }
}

// ---- device-wide scan in one launch: decoupled look-back ----
// Chunks of 4096 values are taken in launch order (an atomic ticket, so a
// chunk only waits on chunks that have started).  Each publishes its sum at
// once, then warp 0 walks back over the status words, 32 at a time, to the
// nearest inclusive prefix (flag 2), publishes its own inclusive prefix and
// the chunk writes its values.  Status word: flag in the high half (1 =
// chunk sum, 2 = inclusive prefix, 3 = failed), value in the low half.  Waits
// are bounded: a walk that gives up sets VS_DERR_WAIT, publishes flag 3 and the
// chunk writes nothing; a walk that meets flag 3 before its nearest inclusive
// prefix fails the same way, so no later chunk writes values built on a
// prefix that was never formed.
constexpr uint32_t SCAN_SPIN_LIMIT = 1u << 22;

__device__ __forceinline__ unsigned long long scan_status_load(unsigned long long* p) {
  cuda::atomic_ref<unsigned long long, cuda::thread_scope_device> r(*p);
  return r.load(cuda::memory_order_acquire);
}
__device__ __forceinline__ void scan_status_store(unsigned long long* p, unsigned long long v) {
  cuda::atomic_ref<unsigned long long, cuda::thread_scope_device> r(*p);
  r.store(v, cuda::memory_order_release);
}

// kGather: the values are src[idx[i]] instead of data[i] (data is only
// written).
template <bool kInclusive, bool kGather>
__global__ void __launch_bounds__(SCAN_THREADS) scan_lookback_kernel(uint32_t* __restrict__ data, uint32_t count,
                                                                     uint32_t nchunks, unsigned long long* status,
                                                                     uint32_t* ticket, unsigned long long* total_dev,
                                                                     uint32_t* err, const uint32_t* __restrict__ src,
                                                                     const uint32_t* __restrict__ idx) {
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_chunk, s_prefix, s_fail;
  const uint32_t tid = threadIdx.x, lane = tid & 31u;
  if (tid == 0) {
    s_chunk = atomicAdd(ticket, 1u);
    s_fail = 0u;
  }
  __syncthreads();
  const uint32_t chunk = s_chunk;
  const uint32_t base = chunk * SCAN_CHUNK + tid * SCAN_ITEMS;
  uint32_t x[SCAN_ITEMS];
  uint32_t sum = 0;
#pragma unroll
  for (uint32_t i = 0; i < SCAN_ITEMS; ++i) {
    x[i] = (base + i < count) ? (kGather ? src[idx[base + i]] : data[base + i]) : 0u;
    sum += x[i];
  }
  uint32_t total;
  const uint32_t in_chunk = block_exclusive_scan(sum, s_warp, &total);
  if (tid == 0) scan_status_store(&status[chunk], ((chunk == 0 ? 2ull : 1ull) << 32) | total);
  if (tid < 32) {
    uint32_t exclusive = 0;
    if (chunk > 0) {
      int64_t hi = (int64_t)chunk - 1;
      uint32_t spins = 0;
      while (true) {
        const int64_t q = hi - (int64_t)lane;
        const unsigned long long st = q >= 0 ? scan_status_load(&status[q]) : (2ull << 32);
        const uint32_t flag = (uint32_t)(st >> 32);
        const uint32_t incl = __ballot_sync(0xffffffffu, flag == 2u);
        const uint32_t pending = __ballot_sync(0xffffffffu, flag == 0u);
        const uint32_t failed = __ballot_sync(0xffffffffu, flag == 3u);
        const uint32_t first = incl ? (uint32_t)(__ffs(incl) - 1) : 32u;
        const uint32_t needed = first >= 31u ? 0xffffffffu : ((2u << first) - 1u);
        if (failed & needed) {  // an earlier chunk gave up: its prefix never formed
          if (lane == 0) {
            atomicOr(err, VS_DERR_WAIT);
            s_fail = 1u;
          }
          break;
        }
        if (pending & needed) {
          if (++spins > SCAN_SPIN_LIMIT) {
            if (lane == 0) {
              atomicOr(err, VS_DERR_WAIT);
              s_fail = 1u;
            }
            break;
          }
          if (spins > 32) __nanosleep(64);
          continue;
        }
        uint32_t part = lane <= first ? (uint32_t)st : 0u;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
        exclusive += part;
        if (first < 32u) break;
        hi -= 32;
      }
      __syncwarp();
      if (lane == 0)
        scan_status_store(&status[chunk], s_fail ? (3ull << 32) : ((2ull << 32) | (exclusive + total)));
    }
    if (lane == 0) {
      s_prefix = exclusive;
      if (chunk == nchunks - 1 && total_dev && !s_fail) *total_dev = (unsigned long long)exclusive + total;
    }
  }
  __syncthreads();
  if (s_fail) return;
  uint32_t run = s_prefix + in_chunk;
#pragma unroll
  for (uint32_t i = 0; i < SCAN_ITEMS; ++i) {
    if (kInclusive) run += x[i];
    if (base + i < count) data[base + i] = run;
    if (!kInclusive) run += x[i];
  }
}

vs_status scan_impl(vs_ctx* ctx, uint32_t* data, uint32_t count, uint64_t* total_dev, bool inclusive,
                    const uint32_t* src = nullptr, const uint32_t* idx = nullptr) {
  if (count == 0) {
    if (total_dev) VS_CUDA(ctx, cudaMemsetAsync(total_dev, 0, 8, ctx->stream));
    return VS_OK;
  }
  const uint32_t chunks = div_up(count, SCAN_CHUNK);
  // one launch: status words (8 B per chunk) and a ticket, cleared first
  const size_t bytes = (size_t)chunks * 8 + 16;
  VS_TRY(vs_ensure(ctx, ctx->scan_sums, bytes));
  unsigned long long* status = (unsigned long long*)ctx->scan_sums.ptr;
  uint32_t* ticket = (uint32_t*)(status + chunks);
  VS_CUDA(ctx, cudaMemsetAsync(status, 0, bytes, ctx->stream));
  unsigned long long* tot = (unsigned long long*)total_dev;
  if (src)
    scan_lookback_kernel<true, true><<<chunks, SCAN_THREADS, 0, ctx->stream>>>(data, count, chunks, status, ticket,
                                                                            tot, ctx->d_err, src, idx);
  else if (inclusive)
    scan_lookback_kernel<true, false><<<chunks, SCAN_THREADS, 0, ctx->stream>>>(data, count, chunks, status, ticket,
                                                                             tot, ctx->d_err, nullptr, nullptr);
  else
    scan_lookback_kernel<false, false><<<chunks, SCAN_THREADS, 0, ctx->stream>>>(data, count, chunks, status,
                                                                              ticket, tot, ctx->d_err, nullptr,
                                                                              nullptr);
  ++ctx->launches;
  return vs_cuda(ctx, cudaGetLastError(), "scan launch");
}

}  // namespace

vs_status scan_inclusive_u32(vs_ctx* ctx, uint32_t* data, uint32_t count, uint64_t* total_dev) {
  return scan_impl(ctx, data, count, total_dev, true);
}

vs_status scan_gather_inclusive_u32(vs_ctx* ctx, uint32_t* out, const uint32_t* src, const uint32_t* idx,
                                    uint32_t count) {
  if (count == 0) return VS_OK;
  return scan_impl(ctx, out, count, nullptr, true, src, idx);
}

uint32_t radix_sort_passes(uint32_t key_bits) { return div_up(key_bits, MAX_DIGIT_BITS); }

vs_status radix_sort_from(vs_ctx* ctx, const uint32_t* keys_in, const uint32_t* vals_in, uint32_t key_sub,
                          uint32_t* a_keys, uint32_t* a_vals, uint32_t* b_keys, uint32_t* b_vals, uint32_t count,
                          uint32_t key_bits, const uint32_t* gather_src, uint32_t* gather_out) {
  if (count == 0 || key_bits == 0) return VS_OK;
  const uint32_t tiles = div_up(count, SORT_TILE);
  const uint32_t passes = radix_sort_passes(key_bits);
  const uint32_t wide = key_bits / passes + (key_bits % passes ? 1u : 0u);  // widest digit
  const size_t hist_n = ((size_t)1 << wide) * tiles;
  if (hist_n > 0xffffffffull) return vs_fail(ctx, VS_ERR_CAPACITY, "radix sort: %u keys exceed the histogram", count);
  VS_TRY(vs_ensure(ctx, ctx->sort_hist, hist_n * sizeof(uint32_t)));
  uint32_t* hist = (uint32_t*)ctx->sort_hist.ptr;
  const uint32_t* kin = keys_in;
  const uint32_t* vin = vals_in;
  uint32_t *kout = a_keys, *vout = a_vals;
  uint32_t shift = 0;
  for (uint32_t p = 0; p < passes; ++p) {
    // the first key_bits % passes passes take one bit more than the rest
    const uint32_t bits = key_bits / passes + (p < key_bits % passes ? 1u : 0u);
    const uint32_t mask = (1u << bits) - 1u;
    const uint32_t sub = p == 0 ? key_sub : 0u;
    const bool last = p + 1 == passes;
    const uint32_t* gs = last ? gather_src : nullptr;
    uint32_t* go = last ? gather_out : nullptr;
    // the table is (mask + 1) x tiles words, within the hist_n allocated above
    if (bits > 8) {
      hist_kernel<9><<<tiles, SORT_THREADS, 0, ctx->stream>>>(kin, count, shift, mask, tiles, hist, sub);
      ++ctx->launches;
      VS_TRY(scan_impl(ctx, hist, (mask + 1u) * tiles, nullptr, false));
      scatter_kernel<9><<<tiles, SORT_THREADS, 0, ctx->stream>>>(kin, vin, kout, vout, count, shift, mask, tiles,
                                                                 hist, sub, gs, go);
    } else {
      hist_kernel<8><<<tiles, SORT_THREADS, 0, ctx->stream>>>(kin, count, shift, mask, tiles, hist, sub);
      ++ctx->launches;
      VS_TRY(scan_impl(ctx, hist, (mask + 1u) * tiles, nullptr, false));
      scatter_kernel<8><<<tiles, SORT_THREADS, 0, ctx->stream>>>(kin, vin, kout, vout, count, shift, mask, tiles,
                                                                 hist, sub, gs, go);
    }
    ++ctx->launches;
    VS_CUDA(ctx, cudaGetLastError());
    kin = kout;
    vin = vout;
    const bool to_b = kout == a_keys;
    kout = to_b ? b_keys : a_keys;
    vout = to_b ? b_vals : a_vals;
    shift += bits;
  }
  return VS_OK;
}

vs_status radix_sort_pairs(vs_ctx* ctx, uint32_t* keys, uint32_t* vals, uint32_t* keys_alt, uint32_t* vals_alt,
                           uint32_t count, uint32_t key_bits, bool* result_in_alt) {
  *result_in_alt = false;
  if (count <= 1 || key_bits == 0) return VS_OK;
  // pass 0 reads (keys, vals) and writes the alternates, pass 1 writes back, ...
  VS_TRY(radix_sort_from(ctx, keys, vals, 0u, keys_alt, vals_alt, keys, vals, count, key_bits, nullptr, nullptr));
  *result_in_alt = (radix_sort_passes(key_bits) & 1u) != 0;
  return VS_OK;
}

// ---------------------------------------------------------------------------
// Sort with file-scope scratch: vs_radix_sort_pairs_static.
//
// For callers that may not allocate device memory during the call: a host
// that runs the sort inside a fixed device-memory budget it manages itself, or
// at a point where an allocation would synchronise the device or be refused.
// Every temporary lives in one statically sized __device__ array that is part
// of the library's device image, so a call launches kernels and issues at most
// two device-to-device copies, nothing else.  Limits and rules:
//   - at most VS_SORT_STATIC_MAX_KEYS (2^20) pairs; larger counts are rejected
//     with VS_ERR_CAPACITY before anything is launched;
//   - the first call on each device looks the array up with
//     cudaGetSymbolAddress (which can load the module); make that first call
//     before any stream capture on that device;
//   - nothing in the array needs to start at zero: every pass writes its whole
//     histogram and all chunk sums before reading them;
//   - the array is shared by every call on a device, so two calls that may run
//     at the same time on the GPU (other streams, other threads) race.
namespace {

constexpr uint32_t STATIC_MAX_KEYS = 1u << 20;
constexpr uint32_t STATIC_TILES = STATIC_MAX_KEYS / SORT_TILE;                 // 512
constexpr uint32_t STATIC_HIST = RADIX * STATIC_TILES;                         // 131072
constexpr uint32_t STATIC_SUMS = (STATIC_HIST + SCAN_CHUNK - 1) / SCAN_CHUNK;  // 32
constexpr size_t STATIC_WORDS = 2ull * STATIC_MAX_KEYS + STATIC_HIST + 64;
static_assert(STATIC_SUMS <= 64, "chunk-sum slots");

static __device__ __align__(256) uint32_t g_sort_scratch[STATIC_WORDS];

std::mutex g_scratch_mu;
uint32_t* g_scratch_ptr[256] = {};

// Device address of g_sort_scratch on ctx's device (looked up once per device,
// with that device current).
vs_status static_scratch(vs_ctx* ctx, uint32_t** out) {
  if (ctx->device < 0 || ctx->device >= 256)
    return vs_fail(ctx, VS_ERR_INVALID, "radix_sort_static: device %d", ctx->device);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[ctx->device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_sort_scratch);
    if (e != cudaSuccess || !p)
      return vs_fail(ctx, VS_ERR_CUDA, "radix_sort_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    g_scratch_ptr[ctx->device] = (uint32_t*)p;
  }
  *out = g_scratch_ptr[ctx->device];
  return VS_OK;
}

// Exclusive scan of `count` words in place with caller-provided chunk sums.
void scan_exclusive_into(vs_ctx* ctx, uint32_t* data, uint32_t count, uint32_t* sums) {
  const uint32_t chunks = div_up(count, SCAN_CHUNK);
  scan_reduce_kernel<<<chunks, SCAN_THREADS, 0, ctx->stream>>>(data, count, sums); ++ctx->launches;
  scan_sums_kernel<<<1, 1024, 0, ctx->stream>>>(sums, chunks, nullptr); ++ctx->launches;
  scan_apply_kernel<false><<<chunks, SCAN_THREADS, 0, ctx->stream>>>(data, count, sums); ++ctx->launches;
}

}  // namespace

extern "C" VS_API vs_status vs_radix_sort_pairs_static(vs_ctx* ctx, uint32_t* keys, uint32_t* values,
                                                       uint32_t count, uint32_t key_bits) {
  if (!ctx) return VS_ERR_INVALID;
  if ((!keys || !values) && count) return vs_fail(ctx, VS_ERR_INVALID, "radix_sort_static: null buffer");
  if (key_bits > 32) return vs_fail(ctx, VS_ERR_INVALID, "radix_sort_static: key_bits %u > 32", key_bits);
  if (count > STATIC_MAX_KEYS)
    return vs_fail(ctx, VS_ERR_CAPACITY, "radix_sort_static: %u pairs exceed the static scratch limit of %u", count,
                   STATIC_MAX_KEYS);
  // the caller's current device is put back on every return
  int prev_device = -1;
  VS_TRY(vs_cuda(ctx, cudaGetDevice(&prev_device), "cudaGetDevice"));
  struct RestoreDevice {
    int dev, cur;
    ~RestoreDevice() {
      if (dev >= 0 && dev != cur) cudaSetDevice(dev);
    }
  } restore{prev_device, ctx->device};
  VS_TRY(vs_cuda(ctx, cudaSetDevice(ctx->device), "cudaSetDevice"));
  uint32_t* scratch = nullptr;
  VS_TRY(static_scratch(ctx, &scratch));
  if (count <= 1 || key_bits == 0) return VS_OK;
  const uint32_t tiles = div_up(count, SORT_TILE);
  uint32_t* keys_alt = scratch;
  uint32_t* vals_alt = scratch + STATIC_MAX_KEYS;
  uint32_t* hist = scratch + 2 * STATIC_MAX_KEYS;
  uint32_t* sums = hist + STATIC_HIST;
  uint32_t *kin = keys, *vin = values, *kout = keys_alt, *vout = vals_alt;
  bool in_alt = false;
  for (uint32_t shift = 0; shift < key_bits; shift += 8) {
    const uint32_t bits = min(8u, key_bits - shift);
    const uint32_t mask = (1u << bits) - 1u;
    hist_kernel<8><<<tiles, SORT_THREADS, 0, ctx->stream>>>(kin, count, shift, mask, tiles, hist); ++ctx->launches;
    scan_exclusive_into(ctx, hist, (mask + 1u) * tiles, sums);
    scatter_kernel<8><<<tiles, SORT_THREADS, 0, ctx->stream>>>(kin, vin, kout, vout, count, shift, mask, tiles, hist); ++ctx->launches;
    VS_TRY(vs_cuda(ctx, cudaGetLastError(), "radix_sort_static launch"));
    uint32_t* t = kin; kin = kout; kout = t;
    t = vin; vin = vout; vout = t;
    in_alt = !in_alt;
  }
  if (in_alt) {
    VS_TRY(vs_cuda(ctx, cudaMemcpyAsync(keys, keys_alt, (size_t)count * 4, cudaMemcpyDeviceToDevice, ctx->stream),
                   "radix_sort_static copy"));
    VS_TRY(vs_cuda(ctx, cudaMemcpyAsync(values, vals_alt, (size_t)count * 4, cudaMemcpyDeviceToDevice, ctx->stream),
                   "radix_sort_static copy"));
  }
  return VS_OK;
}
