// Parallel safetensors I/O.
//
// The reference patches MLX's loader for an adaptive reader thread pool
// (4-16 threads) reading in 128 MiB batches (patches/mlx-swift-loader*.patch;
// MLXLMCommon/Load.swift:60-280 orders span reads per shard). This reader does
// the same natively: the header is parsed by the caller (it is JSON), and the
// tensor payload spans are read with pread() from a pool of threads straight
// into caller-provided (pinned) host memory, 128 MiB per task.
#include <fcntl.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

namespace py = pybind11;

namespace b200host {

static constexpr size_t kChunk = 128ull << 20;

// Returns (header_json, data_start_offset).
std::tuple<std::string, uint64_t> st_read_header(const std::string& path) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error("cannot open " + path);
  uint64_t n = 0;
  if (::pread(fd, &n, 8, 0) != 8) {
    ::close(fd);
    throw std::runtime_error("short read of safetensors header length: " + path);
  }
  if (n > (1ull << 30)) {
    ::close(fd);
    throw std::runtime_error("implausible safetensors header size");
  }
  std::string hdr(n, '\0');
  size_t got = 0;
  while (got < n) {
    ssize_t r = ::pread(fd, &hdr[got], n - got, 8 + got);
    if (r <= 0) {
      ::close(fd);
      throw std::runtime_error("short read of safetensors header: " + path);
    }
    got += (size_t)r;
  }
  ::close(fd);
  return {hdr, 8 + n};
}

static int choose_threads(size_t total_bytes, int requested) {
  if (requested > 0) return requested;
  const unsigned hc = std::max(1u, std::thread::hardware_concurrency());
  // 4 threads for small reads, up to 16 for multi-GB shards
  int t = total_bytes < (1ull << 30) ? 4 : total_bytes < (8ull << 30) ? 8 : 16;
  return std::min<int>(t, (int)hc * 2);
}

// Read spans [(file_offset, nbytes, dst_address)] of one file in parallel.
void st_read_spans(const std::string& path, const std::vector<std::tuple<uint64_t, uint64_t, uintptr_t>>& spans,
                   int threads) {
  struct Task {
    uint64_t off, n;
    char* dst;
  };
  std::vector<Task> tasks;
  size_t total = 0;
  for (auto& s : spans) {
    uint64_t off = std::get<0>(s), n = std::get<1>(s);
    char* dst = reinterpret_cast<char*>(std::get<2>(s));
    total += n;
    for (uint64_t o = 0; o < n; o += kChunk) tasks.push_back({off + o, std::min<uint64_t>(kChunk, n - o), dst + o});
  }
  std::sort(tasks.begin(), tasks.end(), [](const Task& a, const Task& b) { return a.off < b.off; });
  const int nt = std::max(1, std::min<int>(choose_threads(total, threads), (int)tasks.size()));
  std::atomic<size_t> next{0};
  std::atomic<int> err{0};
  std::string errmsg;
  py::gil_scoped_release nogil;
  auto worker = [&]() {
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
      err = 1;
      return;
    }
    while (!err) {
      const size_t i = next.fetch_add(1);
      if (i >= tasks.size()) break;
      const Task& t = tasks[i];
      uint64_t got = 0;
      while (got < t.n) {
        ssize_t r = ::pread(fd, t.dst + got, t.n - got, t.off + got);
        if (r <= 0) {
          err = 2;
          break;
        }
        got += (uint64_t)r;
      }
    }
    ::close(fd);
  };
  std::vector<std::thread> pool;
  for (int i = 0; i < nt; ++i) pool.emplace_back(worker);
  for (auto& th : pool) th.join();
  if (err) throw std::runtime_error("safetensors read failed for " + path);
}

// Write a safetensors file: header JSON (already padded by the caller is not
// required; we pad to 8 bytes) followed by the payload spans (src addresses).
void st_write(const std::string& path, const std::string& header,
              const std::vector<std::tuple<uintptr_t, uint64_t>>& payload) {
  std::string hdr = header;
  while ((hdr.size() % 8) != 0) hdr.push_back(' ');
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) throw std::runtime_error("cannot create " + path);
  uint64_t n = hdr.size();
  std::fwrite(&n, 8, 1, f);
  std::fwrite(hdr.data(), 1, hdr.size(), f);
  for (auto& p : payload) {
    const char* src = reinterpret_cast<const char*>(std::get<0>(p));
    uint64_t len = std::get<1>(p);
    if (len && std::fwrite(src, 1, len, f) != len) {
      std::fclose(f);
      throw std::runtime_error("write failed: " + path);
    }
  }
  std::fclose(f);
}

}  // namespace b200host

void register_safetensors(py::module_& m) {
  using namespace b200host;
  m.def("st_read_header", &st_read_header, py::arg("path"));
  m.def("st_read_spans", &st_read_spans, py::arg("path"), py::arg("spans"), py::arg("threads") = 0);
  m.def("st_write", &st_write, py::arg("path"), py::arg("header"), py::arg("payload"));
}
