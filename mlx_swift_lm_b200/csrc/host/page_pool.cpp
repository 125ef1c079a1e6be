// Host-side paged-KV page pool and prefix block hashing.
//
// PagePool: O(1) free list over a fixed slab of pages with per-page refcounts
// (resident prefix sharing hands the same physical page to several rows) and
// generation counters (a handle taken before a page was freed and reused is
// detected as stale). Poisoned pages are excluded from capacity. Mirrors the
// reference's PagedKVPool (ContinuousBatchingV2/Paged/PagedKVPool.swift:23-1365,
// free list PagedKVFreePages.swift:21, generation checks :934-944, poison
// pages :782-800) on the host; the device slab itself is one torch tensor.
//
// BlockHasher: SHA-256 chain over fixed-size token blocks,
//   h_0 = SHA256(salt || tokens[0:B]), h_i = SHA256(h_{i-1} || tokens[iB:(i+1)B]),
// tokens serialised as little-endian int32, as the reference's prefix cache
// keys blocks (ContinuousBatchingV2/BlockHasher.swift:25-141).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace b200host {

class PagePool {
 public:
  explicit PagePool(int64_t num_pages) : n_(num_pages), ref_(num_pages, 0), gen_(num_pages, 0), poison_(num_pages, 0) {
    free_.reserve(num_pages);
    for (int64_t i = num_pages - 1; i >= 0; --i) free_.push_back(i);
  }

  int64_t num_pages() const { return n_; }
  int64_t num_free() const { return (int64_t)free_.size(); }
  int64_t num_used() const { return n_ - num_poisoned_ - (int64_t)free_.size(); }
  int64_t num_poisoned() const { return num_poisoned_; }

  // Allocate n pages (refcount 1). Throws if not enough free pages.
  std::vector<int64_t> alloc(int64_t n) {
    if (n < 0) throw std::invalid_argument("negative page count");
    if ((int64_t)free_.size() < n) throw std::runtime_error("page pool exhausted");
    std::vector<int64_t> out(n);
    for (int64_t i = 0; i < n; ++i) {
      const int64_t p = free_.back();
      free_.pop_back();
      ref_[p] = 1;
      out[i] = p;
    }
    return out;
  }

  bool can_alloc(int64_t n) const { return (int64_t)free_.size() >= n; }

  void incref(const std::vector<int64_t>& pages) {
    for (auto p : pages) {
      check(p);
      if (ref_[p] <= 0) throw std::runtime_error("incref of a free page");
      ++ref_[p];
    }
  }

  // Drop one reference from each page; pages reaching zero return to the free
  // list (their generation advances). Returns how many pages were freed.
  int64_t decref(const std::vector<int64_t>& pages) {
    int64_t freed = 0;
    for (auto p : pages) {
      check(p);
      if (ref_[p] <= 0) throw std::runtime_error("double free of page " + std::to_string(p));
      if (--ref_[p] == 0) {
        ++gen_[p];
        if (poison_[p]) {
          ++num_poisoned_;
        } else {
          free_.push_back(p);
        }
        ++freed;
      }
    }
    return freed;
  }

  int32_t refcount(int64_t p) const {
    check(p);
    return ref_[p];
  }
  uint32_t generation(int64_t p) const {
    check(p);
    return gen_[p];
  }
  // A (page, generation) handle is valid while the page has not been freed since.
  bool valid(int64_t p, uint32_t gen) const {
    check(p);
    return ref_[p] > 0 && gen_[p] == gen;
  }

  // Poison a page: when its last reference drops it is never reused.
  void poison(int64_t p) {
    check(p);
    if (poison_[p]) return;
    poison_[p] = 1;
    if (ref_[p] == 0) {
      // remove from the free list
      for (size_t i = 0; i < free_.size(); ++i)
        if (free_[i] == p) {
          free_[i] = free_.back();
          free_.pop_back();
          break;
        }
      ++num_poisoned_;
    }
  }

 private:
  void check(int64_t p) const {
    if (p < 0 || p >= n_) throw std::out_of_range("page id out of range: " + std::to_string(p));
  }
  int64_t n_;
  std::vector<int32_t> ref_;
  std::vector<uint32_t> gen_;
  std::vector<uint8_t> poison_;
  std::vector<int64_t> free_;
  int64_t num_poisoned_ = 0;
};

// ---------------------------------------------------------------- SHA-256 (FIPS 180-4)
struct Sha256 {
  uint32_t h[8];
  uint8_t buf[64];
  uint64_t len = 0;
  size_t blen = 0;
  static constexpr uint32_t K[64] = {
      0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
      0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
      0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
      0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
      0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
      0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
      0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
      0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
  Sha256() {
    const uint32_t init[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                              0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    std::memcpy(h, init, sizeof(h));
  }
  static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
  void block(const uint8_t* p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i) w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 |
                                        (uint32_t)p[4 * i + 2] << 8 | (uint32_t)p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      const uint32_t ch = (e & f) ^ (~e & g);
      const uint32_t t1 = hh + S1 + ch + K[i] + w[i];
      const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
      const uint32_t t2 = S0 + mj;
      hh = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  void update(const uint8_t* p, size_t n) {
    len += n;
    while (n > 0) {
      const size_t take = std::min(n, 64 - blen);
      std::memcpy(buf + blen, p, take);
      blen += take;
      p += take;
      n -= take;
      if (blen == 64) {
        block(buf);
        blen = 0;
      }
    }
  }
  std::string digest() {
    const uint64_t bits = len * 8;
    const uint8_t pad = 0x80;
    update(&pad, 1);
    const uint8_t z = 0;
    while (blen != 56) update(&z, 1);
    uint8_t lb[8];
    for (int i = 0; i < 8; ++i) lb[i] = (uint8_t)(bits >> (56 - 8 * i));
    update(lb, 8);
    std::string out(32, '\0');
    for (int i = 0; i < 8; ++i)
      for (int j = 0; j < 4; ++j) out[4 * i + j] = (char)(h[i] >> (24 - 8 * j));
    return out;
  }
};
constexpr uint32_t Sha256::K[64];

py::bytes sha256(const std::string& data) {
  Sha256 s;
  s.update(reinterpret_cast<const uint8_t*>(data.data()), data.size());
  return py::bytes(s.digest());
}

// Chain hashes of the full blocks of `tokens` (a trailing partial block is not hashed).
std::vector<py::bytes> block_hashes(const std::vector<int32_t>& tokens, int block_size, const std::string& salt) {
  if (block_size <= 0) throw std::invalid_argument("block_size must be positive");
  std::vector<py::bytes> out;
  std::string prev = salt;
  const size_t nb = tokens.size() / block_size;
  for (size_t b = 0; b < nb; ++b) {
    Sha256 s;
    s.update(reinterpret_cast<const uint8_t*>(prev.data()), prev.size());
    for (int i = 0; i < block_size; ++i) {
      const int32_t t = tokens[b * block_size + i];
      uint8_t le[4] = {(uint8_t)t, (uint8_t)(t >> 8), (uint8_t)(t >> 16), (uint8_t)(t >> 24)};
      s.update(le, 4);
    }
    prev = s.digest();
    out.emplace_back(py::bytes(prev));
  }
  return out;
}

}  // namespace b200host

void register_page_pool(py::module_& m) {
  using namespace b200host;
  py::class_<PagePool>(m, "PagePool")
      .def(py::init<int64_t>(), py::arg("num_pages"))
      .def_property_readonly("num_pages", &PagePool::num_pages)
      .def_property_readonly("num_free", &PagePool::num_free)
      .def_property_readonly("num_used", &PagePool::num_used)
      .def_property_readonly("num_poisoned", &PagePool::num_poisoned)
      .def("alloc", &PagePool::alloc, py::arg("n"))
      .def("can_alloc", &PagePool::can_alloc)
      .def("incref", &PagePool::incref)
      .def("decref", &PagePool::decref)
      .def("refcount", &PagePool::refcount)
      .def("generation", &PagePool::generation)
      .def("valid", &PagePool::valid)
      .def("poison", &PagePool::poison);
  m.def("sha256", &sha256);
  m.def("block_hashes", &block_hashes, py::arg("tokens"), py::arg("block_size"), py::arg("salt") = std::string());
}
