// Host-side pieces of the C ABI: status strings, the blake2b-64 block key and the planners that
// turn parameter blocks into launch segments. No device work happens here.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include <atomic>

#include "muzo_b200.h"

namespace muzo {

static thread_local int g_last_cuda_error = 0;

void set_last_cuda_error(cudaError_t err) { g_last_cuda_error = static_cast<int>(err); }

int device_sm_count() {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int v = cached[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    cached[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// ------------------------------------------------------------------ BLAKE2b (RFC 7693)
// Unkeyed BLAKE2b with an 8-byte digest, written from the RFC's description: the SHA-512
// initial vector, the 12-round message schedule SIGMA and the G mixing function with rotation
// distances 32, 24, 16 and 63.
namespace {

const uint64_t kBlakeIV[8] = {
    0x6a09e667f3bcc908ULL, 0xbb67ae8584caa73bULL, 0x3c6ef372fe94f82bULL, 0xa54ff53a5f1d36f1ULL,
    0x510e527fade682d1ULL, 0x9b05688c2b3e6c1fULL, 0x1f83d9abfb41bd6bULL, 0x5be0cd19137e2179ULL};

const uint8_t kSigma[12][16] = {
    {0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15},
    {14, 10, 4, 8, 9, 15, 13, 6, 1, 12, 0, 2, 11, 7, 5, 3},
    {11, 8, 12, 0, 5, 2, 15, 13, 10, 14, 3, 6, 7, 1, 9, 4},
    {7, 9, 3, 1, 13, 12, 11, 14, 2, 6, 5, 10, 4, 0, 15, 8},
    {9, 0, 5, 7, 2, 4, 10, 15, 14, 1, 11, 12, 6, 8, 3, 13},
    {2, 12, 6, 10, 0, 11, 8, 3, 4, 13, 7, 5, 15, 14, 1, 9},
    {12, 5, 1, 15, 14, 13, 4, 10, 0, 7, 6, 3, 9, 2, 8, 11},
    {13, 11, 7, 14, 12, 1, 3, 9, 5, 0, 15, 4, 8, 6, 2, 10},
    {6, 15, 14, 9, 11, 3, 0, 8, 12, 2, 13, 7, 1, 4, 10, 5},
    {10, 2, 8, 4, 7, 6, 1, 5, 15, 11, 9, 14, 3, 12, 13, 0},
    {0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15},
    {14, 10, 4, 8, 9, 15, 13, 6, 1, 12, 0, 2, 11, 7, 5, 3}};

inline uint64_t rotr64(uint64_t x, int n) { return (x >> n) | (x << (64 - n)); }

inline void mix(uint64_t* v, int a, int b, int c, int d, uint64_t x, uint64_t y) {
  v[a] = v[a] + v[b] + x;
  v[d] = rotr64(v[d] ^ v[a], 32);
  v[c] = v[c] + v[d];
  v[b] = rotr64(v[b] ^ v[c], 24);
  v[a] = v[a] + v[b] + y;
  v[d] = rotr64(v[d] ^ v[a], 16);
  v[c] = v[c] + v[d];
  v[b] = rotr64(v[b] ^ v[c], 63);
}

void compress(uint64_t h[8], const uint8_t block[128], uint64_t bytes_so_far, bool last) {
  uint64_t m[16];
  for (int i = 0; i < 16; ++i) {
    uint64_t w = 0;
    for (int b = 7; b >= 0; --b) w = (w << 8) | block[8 * i + b];
    m[i] = w;
  }
  uint64_t v[16];
  for (int i = 0; i < 8; ++i) { v[i] = h[i]; v[i + 8] = kBlakeIV[i]; }
  v[12] ^= bytes_so_far;  // low word of the 128-bit byte counter (messages here are short)
  if (last) v[14] = ~v[14];
  for (int r = 0; r < 12; ++r) {
    const uint8_t* s = kSigma[r];
    mix(v, 0, 4, 8, 12, m[s[0]], m[s[1]]);
    mix(v, 1, 5, 9, 13, m[s[2]], m[s[3]]);
    mix(v, 2, 6, 10, 14, m[s[4]], m[s[5]]);
    mix(v, 3, 7, 11, 15, m[s[6]], m[s[7]]);
    mix(v, 0, 5, 10, 15, m[s[8]], m[s[9]]);
    mix(v, 1, 6, 11, 12, m[s[10]], m[s[11]]);
    mix(v, 2, 7, 8, 13, m[s[12]], m[s[13]]);
    mix(v, 3, 4, 9, 14, m[s[14]], m[s[15]]);
  }
  for (int i = 0; i < 8; ++i) h[i] ^= v[i] ^ v[i + 8];
}

uint64_t blake2b_64(const uint8_t* data, size_t len) {
  uint64_t h[8];
  for (int i = 0; i < 8; ++i) h[i] = kBlakeIV[i];
  h[0] ^= 0x01010000ULL ^ 8ULL;  // depth 1, fanout 1, no key, 8-byte digest
  uint8_t block[128];
  size_t off = 0;
  while (len - off > 128) {
    std::memcpy(block, data + off, 128);
    off += 128;
    compress(h, block, off, false);
  }
  std::memset(block, 0, sizeof(block));
  std::memcpy(block, data + off, len - off);
  compress(h, block, len, true);
  return h[0];  // the digest is the little-endian bytes of h[0]
}

// ------------------------------------------------------------------ torch launch emulation
// torch's CUDA generator fills a contiguous noise tensor with one grid-stride launch of 256-thread
// blocks, grid = min(ceil(numel/256), SMs * (maxThreadsPerSM/256)), each thread drawing one
// Philox block (4 words) per loop trip. The generator offset advances by
// ((numel-1)/(threads*4)+1)*4 per launch. A tensor whose byte offsets overflow int32 is first
// charged for the whole tensor and then split in halves (low half first) until each piece fits;
// every piece is a launch of its own with its own offset.

struct Launch {
  int64_t start, count;
  uint32_t threads;
  uint64_t offset;
};

uint32_t launch_threads(int64_t numel, int sm_count, int max_threads_per_sm) {
  int64_t blocks = (numel + 255) / 256;
  int64_t cap = static_cast<int64_t>(sm_count) * (max_threads_per_sm / 256);
  if (blocks > cap) blocks = cap;
  return static_cast<uint32_t>(blocks * 256);
}

uint64_t launch_offset_increment(int64_t numel, uint32_t threads) {
  uint64_t inc = static_cast<uint64_t>((numel - 1) / (static_cast<int64_t>(threads) * 4) + 1) * 4;
  return (inc + 3) / 4 * 4;
}

bool fits_32bit(int64_t numel, int elem_size) {
  const int64_t kMax = 2147483647LL;
  if (numel > kMax) return false;
  return 1 + (numel - 1) * static_cast<int64_t>(elem_size) <= kMax;
}

void split_leaves(int64_t start, int64_t count, int elem_size, std::vector<std::pair<int64_t, int64_t>>& out) {
  if (fits_32bit(count, elem_size)) { out.emplace_back(start, count); return; }
  int64_t first = count / 2;
  split_leaves(start, first, elem_size, out);
  split_leaves(start + first, count - first, elem_size, out);
}

void plan_noise_launches(int64_t numel, int elem_size, int sm_count, int max_threads_per_sm,
                         std::vector<Launch>& out) {
  if (numel <= 0) return;
  uint64_t gen_offset = 0;
  uint32_t thr = launch_threads(numel, sm_count, max_threads_per_sm);
  uint64_t top_offset = gen_offset;
  gen_offset += launch_offset_increment(numel, thr);
  if (fits_32bit(numel, elem_size)) {
    out.push_back({0, numel, thr, top_offset});
    return;
  }
  std::vector<std::pair<int64_t, int64_t>> leaves;
  split_leaves(0, numel, elem_size, leaves);
  for (auto& lf : leaves) {
    uint32_t t = launch_threads(lf.second, sm_count, max_threads_per_sm);
    out.push_back({lf.first, lf.second, t, gen_offset});
    gen_offset += launch_offset_increment(lf.second, t);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace muzo

using namespace muzo;

extern "C" {

int muzo_abi_version(void) { return MUZO_ABI_VERSION; }

int muzo_last_cuda_error(void) { return g_last_cuda_error; }

const char* muzo_status_string(int status) {
  switch (status) {
    case MUZO_OK: return "ok";
    case MUZO_ERR_ARG: return "invalid argument";
    case MUZO_ERR_DTYPE: return "unsupported dtype";
    case MUZO_ERR_ALIGN: return "pointer or leading dimension not 16-byte aligned";
    case MUZO_ERR_CUDA: return "CUDA runtime error";
    case MUZO_ERR_CAPACITY: return "table capacity exceeded";
    case MUZO_ERR_UNSUPPORTED: return "unsupported shape or device";
    default: return "unknown status";
  }
}

int muzo_hash64_seed(uint64_t base_seed, const char* name, const int64_t* shape, int ndim,
                     int64_t block_index, uint64_t* key_out) {
  if (name == nullptr || key_out == nullptr || ndim < 0 || (ndim > 0 && shape == nullptr))
    return MUZO_ERR_ARG;
  // payload = "<seed>|<name>|<d0>,<d1>,...|<block>" (prng.py:27-34)
  std::string payload = std::to_string(base_seed);
  payload += '|';
  payload += name;
  payload += '|';
  for (int i = 0; i < ndim; ++i) {
    if (i) payload += ',';
    payload += std::to_string(static_cast<long long>(shape[i]));
  }
  payload += '|';
  payload += std::to_string(static_cast<long long>(block_index));
  uint64_t h = blake2b_64(reinterpret_cast<const uint8_t*>(payload.data()), payload.size());
  *key_out = h & ((1ULL << 63) - 1);
  return MUZO_OK;
}

int muzo_plan_segments(const int64_t* numels, void* const* params, void* const* outs, int nblocks,
                       int dist, int sm_count, int max_threads_per_sm, muzo_segment* segs,
                       int capacity, int* nsegs, int64_t* total_items) {
  if (numels == nullptr || params == nullptr || nsegs == nullptr || total_items == nullptr ||
      nblocks < 0 || sm_count <= 0 || max_threads_per_sm < 256 ||
      (dist != MUZO_NORMAL && dist != MUZO_RADEMACHER))
    return MUZO_ERR_ARG;
  // Noise tensor element size: fp32 for randn, int8 for randint (prng.py:63-79).
  const int elem_size = dist == MUZO_NORMAL ? 4 : 1;
  int n = 0;
  int64_t items = 0;
  std::vector<Launch> launches;
  for (int b = 0; b < nblocks; ++b) {
    if (numels[b] < 0) return MUZO_ERR_ARG;
    launches.clear();
    plan_noise_launches(numels[b], elem_size, sm_count, max_threads_per_sm, launches);
    for (const Launch& l : launches) {
      if (n >= capacity) return MUZO_ERR_CAPACITY;
      if (segs != nullptr) {
        muzo_segment& s = segs[n];
        std::memset(&s, 0, sizeof(s));
        s.param = params[b] ? static_cast<char*>(params[b]) : nullptr;
        s.out = (outs && outs[b]) ? static_cast<char*>(outs[b]) : nullptr;
        s.numel = l.count;
        s.item_begin = items;
        s.philox_offset = l.offset;
        s.threads = l.threads;
        s.block_index = b;
        s.elem_start = l.start;
      }
      // one item = 8 consecutive threads x 4 Philox words: ceil(count / (4*threads)) trips
      int64_t trips = (l.count - 1) / (static_cast<int64_t>(l.threads) * 4) + 1;
      int64_t seg_items = trips * (l.threads / 8);
      seg_items = (seg_items + MUZO_ITEMS_PER_CTA - 1) / MUZO_ITEMS_PER_CTA * MUZO_ITEMS_PER_CTA;
      items += seg_items;
      ++n;
    }
  }
  *nsegs = n;
  *total_items = items;
  return MUZO_OK;
}

int muzo_plan_linear(const int64_t* numels, void* const* params, void* const* outs, int nblocks,
                     muzo_segment* segs, int capacity, int* nsegs, int64_t* total_items) {
  if (numels == nullptr || params == nullptr || nsegs == nullptr || total_items == nullptr ||
      nblocks < 0)
    return MUZO_ERR_ARG;
  int64_t items = 0;
  if (nblocks > capacity && segs != nullptr) return MUZO_ERR_CAPACITY;
  for (int b = 0; b < nblocks; ++b) {
    if (numels[b] < 0) return MUZO_ERR_ARG;
    if (segs != nullptr) {
      muzo_segment& s = segs[b];
      std::memset(&s, 0, sizeof(s));
      s.param = params[b];
      s.out = outs ? outs[b] : nullptr;
      s.numel = numels[b];
      s.item_begin = items;
      s.block_index = b;
    }
    int64_t seg_items = (numels[b] + 7) / 8;
    seg_items = (seg_items + MUZO_ITEMS_PER_CTA - 1) / MUZO_ITEMS_PER_CTA * MUZO_ITEMS_PER_CTA;
    items += seg_items;
  }
  *nsegs = nblocks;
  *total_items = items;
  return MUZO_OK;
}

}  // extern "C"
