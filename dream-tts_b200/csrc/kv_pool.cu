// The paged KV cache's page allocator behind the C ABI: the reference keeps one contiguous cache
// per lane and narrows it when lanes are shed (crates/qwen3tts/src/qwen3.rs:122-212), and
// broadcast-copies a shared prompt prefix into every lane (qwen3.rs:261-284); here a lane owns a
// row of a block table of fixed-size pages drawn from one pool, a shared prefix's full pages are
// shared between lanes by reference count, and only a partly filled last page is copied.
//
// Host-side bookkeeping (free list, per-lane page lists, reference counts) lives in this object;
// the device sees the block table and the positions, which every admission updates with a
// stream-ordered launch (the host never waits). One pool per group of lanes and per host thread (not thread-safe, as
// the reference's dispatcher is single-threaded).
#include <cuda_runtime.h>

#include <algorithm>
#include <string>
#include <vector>

#include "tts_cuda.h"
#include "tts_internal.h"

// the runtime's error reporting and context accessor (runtime.cu)
namespace rt {
tts_status fail(tts_status s, const std::string& msg);
tts_status cuda_status(cudaError_t e, const char* op);
int ctx_device(const tts_ctx* c);
}  // namespace rt

using rt::cuda_status;
using rt::fail;

struct tts_kv_pool {
  tts_kv_pool_desc d{};
  int device = 0;
  bool owns_pages = false, owns_table = false, owns_positions = false;
  std::vector<int> free;                 // a stack: the next page is free.back()
  std::vector<std::vector<int>> owned;   // pages of each lane, in block-table order
  std::vector<int> refs;                 // lanes holding each page
  size_t page_bytes = 0;                 // one page of one layer, K or V
};

namespace {

struct Guard {
  int prev = -1;
  explicit Guard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~Guard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

void release_lane(tts_kv_pool* p, int lane) {
  for (int pg : p->owned[lane])
    if (--p->refs[pg] == 0) p->free.push_back(pg);
  p->owned[lane].clear();
}

// A run of a block-table row, passed by value in the kernel's parameters: the launch copies
// it, so admissions stay stream-ordered without a host staging buffer or a host wait.
constexpr int kRowChunk = 480;
struct RowChunk {
  int n;
  int pages[kRowChunk];
};

__global__ void set_row_kernel(int* row, RowChunk c, int* position, int length) {
  for (int i = threadIdx.x; i < c.n; i += blockDim.x) row[i] = c.pages[i];
  if (position && threadIdx.x == 0) *position = length;
}

// Writes the lane's block-table row (unused entries 0) and its position, on `stream`.
tts_status write_row(tts_kv_pool* p, int lane, int length, void* stream, const char* op) {
  const int mb = p->d.max_blocks;
  int* row = p->d.block_table + size_t(lane) * mb;
  const auto& o = p->owned[lane];
  for (int c0 = 0; c0 < mb; c0 += kRowChunk) {
    RowChunk c{};
    c.n = std::min(kRowChunk, mb - c0);
    for (int i = 0; i < c.n; ++i) c.pages[i] = c0 + i < int(o.size()) ? o[c0 + i] : 0;
    const bool last = c0 + kRowChunk >= mb;
    set_row_kernel<<<1, 128, 0, S(stream)>>>(row + c0, c, last ? p->d.positions + lane : nullptr,
                                             length);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, op);
  }
  return TTS_OK;
}

tts_status check_lane(const tts_kv_pool* p, int lane, const char* op) {
  if (!p) return fail(TTS_ERR_INVALID_ARG, std::string(op) + ": pool is NULL");
  if (lane < 0 || lane >= p->d.max_lanes)
    return fail(TTS_ERR_INVALID_ARG, std::string(op) + ": lane " + std::to_string(lane) +
                                         " outside 0.." + std::to_string(p->d.max_lanes - 1));
  return TTS_OK;
}

}  // namespace

extern "C" {

tts_status tts_kv_pool_create(tts_ctx* ctx, const tts_kv_pool_desc* desc, tts_kv_pool** out) {
  if (!ctx || !desc || !out) return fail(TTS_ERR_INVALID_ARG, "kv_pool_create: NULL argument");
  const tts_kv_pool_desc& d = *desc;
  if (d.layers < 1 || d.n_kv < 1 || d.head_dim < 1 || d.block_size < 1 || d.num_blocks < 1 ||
      d.max_lanes < 1 || d.max_blocks < 1)
    return fail(TTS_ERR_INVALID_ARG, "kv_pool_create: every size must be >= 1");
  if ((d.k_pages == nullptr) != (d.v_pages == nullptr))
    return fail(TTS_ERR_INVALID_ARG, "kv_pool_create: give both page pools or neither");
  const int device = rt::ctx_device(ctx);
  Guard g(device);
  auto* p = new tts_kv_pool();
  p->d = d;
  p->device = device;
  p->page_bytes = size_t(d.n_kv) * d.block_size * d.head_dim * 2;
  const size_t pool_bytes = p->page_bytes * d.num_blocks * d.layers;
  cudaError_t e = cudaSuccess;
  if (!d.k_pages) {
    e = cudaMalloc(&p->d.k_pages, pool_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&p->d.v_pages, pool_bytes);
    if (e == cudaSuccess) e = cudaMemset(p->d.k_pages, 0, pool_bytes);
    if (e == cudaSuccess) e = cudaMemset(p->d.v_pages, 0, pool_bytes);
    p->owns_pages = true;
  }
  if (e == cudaSuccess && !d.block_table) {
    e = cudaMalloc(reinterpret_cast<void**>(&p->d.block_table),
                   size_t(d.max_lanes) * d.max_blocks * sizeof(int));
    if (e == cudaSuccess)
      e = cudaMemset(p->d.block_table, 0, size_t(d.max_lanes) * d.max_blocks * sizeof(int));
    p->owns_table = true;
  }
  if (e == cudaSuccess && !d.positions) {
    e = cudaMalloc(reinterpret_cast<void**>(&p->d.positions), size_t(d.max_lanes) * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(p->d.positions, 0, size_t(d.max_lanes) * sizeof(int));
    p->owns_positions = true;
  }
  if (e != cudaSuccess) {
    tts_kv_pool_destroy(p);
    return cuda_status(e, "kv_pool_create");
  }
  p->free.reserve(size_t(d.num_blocks));
  for (int i = d.num_blocks - 1; i >= 0; --i) p->free.push_back(i);  // page 0 is taken first
  p->owned.assign(size_t(d.max_lanes), {});
  p->refs.assign(size_t(d.num_blocks), 0);
  *out = p;
  return TTS_OK;
}

tts_status tts_kv_pool_destroy(tts_kv_pool* p) {
  if (!p) return TTS_OK;
  Guard g(p->device);
  if (p->owns_pages) {
    cudaFree(p->d.k_pages);
    cudaFree(p->d.v_pages);
  }
  if (p->owns_table) cudaFree(p->d.block_table);
  if (p->owns_positions) cudaFree(p->d.positions);
  delete p;
  return TTS_OK;
}

tts_status tts_kv_pool_admit(tts_kv_pool* p, int lane, int capacity, int length, void* stream) {
  tts_status st = check_lane(p, lane, "kv_pool_admit");
  if (st != TTS_OK) return st;
  if (capacity < 1 || length < 0 || length > capacity)
    return fail(TTS_ERR_INVALID_ARG, "kv_pool_admit: need 0 <= length <= capacity, capacity >= 1");
  const int need = (capacity + p->d.block_size - 1) / p->d.block_size;
  if (need > p->d.max_blocks)
    return fail(TTS_ERR_INVALID_ARG, "kv_pool_admit: lane needs " + std::to_string(need) +
                                         " pages, the table holds " +
                                         std::to_string(p->d.max_blocks));
  release_lane(p, lane);
  if (size_t(need) > p->free.size())
    return fail(TTS_ERR_OOM, "kv_pool_admit: KV pool exhausted (" + std::to_string(need) +
                                 " pages wanted, " + std::to_string(p->free.size()) + " free)");
  for (int i = 0; i < need; ++i) {
    const int pg = p->free.back();
    p->free.pop_back();
    p->refs[pg] = 1;
    p->owned[lane].push_back(pg);
  }
  Guard g(p->device);
  return write_row(p, lane, length, stream, "kv_pool_admit");
}

tts_status tts_kv_pool_admit_pages(tts_kv_pool* p, int lane, const int* pages, int n, int length,
                                   void* stream) {
  tts_status st = check_lane(p, lane, "kv_pool_admit_pages");
  if (st != TTS_OK) return st;
  if (!pages || n < 1 || n > p->d.max_blocks || length < 0 || length > n * p->d.block_size)
    return fail(TTS_ERR_INVALID_ARG,
                "kv_pool_admit_pages: 1 <= n <= max_blocks pages, length within them");
  release_lane(p, lane);
  for (int i = 0; i < n; ++i) {
    const int pg = pages[i];
    if (pg < 0 || pg >= p->d.num_blocks || p->refs[pg] != 0 ||
        std::count(pages, pages + i, pg))
      return fail(TTS_ERR_INVALID_ARG, "kv_pool_admit_pages: page " + std::to_string(pg) +
                                           " is not a free page of the pool");
  }
  for (int i = 0; i < n; ++i) {
    const int pg = pages[i];
    p->free.erase(std::find(p->free.begin(), p->free.end(), pg));
    p->refs[pg] = 1;
    p->owned[lane].push_back(pg);
  }
  Guard g(p->device);
  return write_row(p, lane, length, stream, "kv_pool_admit_pages");
}

tts_status tts_kv_pool_share_prefix(tts_kv_pool* p, int src, int lane, int length, int capacity,
                                    void* stream) {
  tts_status st = check_lane(p, lane, "kv_pool_share_prefix");
  if (st == TTS_OK) st = check_lane(p, src, "kv_pool_share_prefix");
  if (st != TTS_OK) return st;
  const int bs = p->d.block_size;
  const int need = (capacity + bs - 1) / bs;
  if (src == lane || need > p->d.max_blocks || length < 0 || length > capacity)
    return fail(TTS_ERR_INVALID_ARG,
                "kv_pool_share_prefix: another lane, capacity within the block table, "
                "0 <= length <= capacity");
  const int full = length / bs, part = length % bs;
  const std::vector<int> src_pages = p->owned[src];
  if (int(src_pages.size()) < full + (part ? 1 : 0))
    return fail(TTS_ERR_INVALID_ARG, "kv_pool_share_prefix: the source lane holds fewer pages "
                                     "than the prefix");
  release_lane(p, lane);
  if (size_t(need - full) > p->free.size())
    return fail(TTS_ERR_OOM, "kv_pool_share_prefix: KV pool exhausted");
  for (int i = 0; i < full; ++i) {
    ++p->refs[src_pages[i]];
    p->owned[lane].push_back(src_pages[i]);
  }
  std::vector<int> fresh;
  for (int i = full; i < need; ++i) {
    const int pg = p->free.back();
    p->free.pop_back();
    p->refs[pg] = 1;
    p->owned[lane].push_back(pg);
    fresh.push_back(pg);
  }
  Guard g(p->device);
  if (part) {
    // the partly filled page: this lane writes its own rows after the prefix, so it gets a copy
    // (every layer's K and V page)
    for (int l = 0; l < p->d.layers; ++l)
      for (void* base : {p->d.k_pages, p->d.v_pages}) {
        char* b = static_cast<char*>(base) + size_t(l) * p->d.num_blocks * p->page_bytes;
        const cudaError_t e =
            cudaMemcpyAsync(b + size_t(fresh[0]) * p->page_bytes,
                            b + size_t(src_pages[full]) * p->page_bytes, p->page_bytes,
                            cudaMemcpyDeviceToDevice, S(stream));
        if (e != cudaSuccess) return cuda_status(e, "kv_pool_share_prefix");
      }
  }
  return write_row(p, lane, length, stream, "kv_pool_share_prefix");
}

tts_status tts_kv_pool_release(tts_kv_pool* p, int lane) {
  tts_status st = check_lane(p, lane, "kv_pool_release");
  if (st != TTS_OK) return st;
  release_lane(p, lane);
  return TTS_OK;
}

int tts_kv_pool_free_pages(const tts_kv_pool* p) { return p ? int(p->free.size()) : -1; }

tts_status tts_kv_pool_lane_pages(const tts_kv_pool* p, int lane, int* pages, int cap, int* n) {
  tts_status st = check_lane(p, lane, "kv_pool_lane_pages");
  if (st != TTS_OK) return st;
  if (!n || (cap > 0 && !pages)) return fail(TTS_ERR_INVALID_ARG, "kv_pool_lane_pages: NULL");
  const auto& o = p->owned[lane];
  *n = int(o.size());
  for (int i = 0; i < cap && i < int(o.size()); ++i) pages[i] = o[i];
  return TTS_OK;
}

int tts_kv_pool_page_refs(const tts_kv_pool* p, int page) {
  if (!p || page < 0 || page >= p->d.num_blocks) return -1;
  return p->refs[page];
}

tts_status tts_kv_pool_state(const tts_kv_pool* p, int lanes, int max_span,
                             tts_decode_state* out) {
  if (!p || !out) return fail(TTS_ERR_INVALID_ARG, "kv_pool_state: NULL argument");
  if (lanes < 1 || lanes > p->d.max_lanes)
    return fail(TTS_ERR_INVALID_ARG, "kv_pool_state: lanes must be in 1..max_lanes");
  out->lanes = lanes;
  out->positions = p->d.positions;
  out->block_table = p->d.block_table;
  out->max_blocks = p->d.max_blocks;
  out->block_size = p->d.block_size;
  out->num_blocks = p->d.num_blocks;
  out->k_pages = p->d.k_pages;
  out->v_pages = p->d.v_pages;
  out->max_span = max_span > 0 ? max_span : p->d.max_blocks * p->d.block_size;
  return TTS_OK;
}

}  // extern "C"
