// index_io.cpp -- DiskANN-layout index files on the host (see index_io.h).
#include "index_io.h"

#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "quiver_b200.h"

namespace qv {
namespace fs = std::filesystem;

int64_t element_size(int32_t data_type) { return data_type == QV_FLOAT ? 4 : 1; }

static bool has_suffix(const std::string& v, const std::string& s) {
  return v.size() >= s.size() && v.compare(v.size() - s.size(), s.size(), s) == 0;
}

// Regular files (symlinks followed) in `dir` ending in `suffix`, sorted
// (index_discovery.hpp:36-52).
static std::vector<std::string> suffix_matches(const std::string& dir, const std::string& suffix) {
  std::vector<std::string> out;
  std::error_code ec;
  for (const auto& e : fs::directory_iterator(dir, ec)) {
    if (!fs::is_regular_file(e.path(), ec)) continue;
    if (has_suffix(e.path().filename().string(), suffix)) out.push_back(e.path().string());
  }
  std::sort(out.begin(), out.end());
  return out;
}

static void require_dir(const std::string& dir) {
  std::error_code ec;
  if (!fs::is_directory(dir, ec))
    throw IoError(QV_ERR_IO, "--index-dir '" + dir + "' does not exist or is not a directory");
}

static std::string join(const std::vector<std::string>& v) {
  std::string s;
  for (size_t i = 0; i < v.size(); ++i) s += (i ? ", " : "") + v[i];
  return s;
}

// index_discovery.hpp:57-78
std::string find_index_file(const std::string& index_dir) {
  require_dir(index_dir);
  const auto m = suffix_matches(index_dir, "_disk.index");
  if (m.size() == 1) return m.front();
  if (m.size() > 1)
    throw IoError(QV_ERR_IO, "Multiple *_disk.index candidates found in " + index_dir + ": " + join(m));
  const fs::path fb = fs::path(index_dir) / "disk.index";
  std::error_code ec;
  if (fs::is_regular_file(fb, ec)) return fb.string();
  throw IoError(QV_ERR_IO, "No *_disk.index or disk.index found in " + index_dir);
}

// index_discovery.hpp:80-103
std::string find_pq_prefix(const std::string& index_dir) {
  require_dir(index_dir);
  const auto m = suffix_matches(index_dir, "_pq_pivots.bin");
  if (m.size() == 1) return m.front().substr(0, m.front().size() - std::string("_pivots.bin").size());
  if (m.size() > 1)
    throw IoError(QV_ERR_IO, "Multiple *_pq_pivots.bin candidates found in " + index_dir + ": " + join(m));
  const std::string fb = (fs::path(index_dir) / "pq").string();
  std::error_code ec;
  if (fs::exists(fb + "_pivots.bin", ec)) return fb;
  throw IoError(QV_ERR_IO, "No PQ pivot files found in " + index_dir);
}

// index_discovery.hpp:105-115
std::string find_nav_dir(const std::string& index_dir) {
  std::error_code ec;
  if (fs::exists(fs::path(index_dir) / "nav_index", ec)) return index_dir;
  if (fs::exists(fs::path(index_dir) / "nav" / "nav_index", ec))
    return (fs::path(index_dir) / "nav").string();
  return "";
}

struct File {
  FILE* f = nullptr;
  explicit File(const std::string& p) : f(std::fopen(p.c_str(), "rb")) {
    if (!f) throw IoError(QV_ERR_IO, "Cannot open file: " + p + " (" + std::strerror(errno) + ")");
  }
  ~File() { if (f) std::fclose(f); }
  void seek(int64_t off, const std::string& what) {
    if (std::fseek(f, static_cast<long>(off), SEEK_SET) != 0)
      throw IoError(QV_ERR_IO, "seek failed in " + what);
  }
  void read(void* dst, size_t n, const std::string& what) {
    if (n && std::fread(dst, 1, n, f) != n) throw IoError(QV_ERR_BAD_INDEX, "truncated " + what);
  }
};

// metadata.hpp:15-72
Layout parse_disk_index_header(const std::string& path, int32_t data_type) {
  File f(path);
  uint32_t nr = 0, nc = 0;
  f.read(&nr, 4, path);
  f.read(&nc, 4, path);
  uint64_t v[8];
  f.read(v, sizeof(v), path);
  Layout L;
  L.data_type = data_type;
  L.num_points = static_cast<int64_t>(v[0]);
  L.dim = static_cast<int64_t>(v[1]);
  L.medoid = static_cast<int64_t>(v[2]);
  L.node_size = static_cast<int64_t>(v[3]);
  L.nodes_per_page = static_cast<int64_t>(v[4]);
  const int64_t es = element_size(data_type);
  L.data_size = L.dim * es;
  if (L.dim <= 0 || L.node_size < L.data_size + 8 || L.nodes_per_page <= 0)
    throw IoError(QV_ERR_BAD_INDEX, "invalid disk index header in " + path);
  L.max_degree = (L.node_size - L.data_size) / 4 - 1;
  L.num_pages = (L.num_points + L.nodes_per_page - 1) / L.nodes_per_page;
  return L;
}

// read_bin of pq_search.cu:185-199: int32 npts, int32 ndims, then data.
template <class T>
static std::vector<T> read_bin(File& f, int64_t offset, int32_t& npts, int32_t& ndims,
                               const std::string& what) {
  f.seek(offset, what);
  f.read(&npts, 4, what);
  f.read(&ndims, 4, what);
  if (npts < 0 || ndims < 0) throw IoError(QV_ERR_BAD_INDEX, "negative shape in " + what);
  std::vector<T> out(static_cast<size_t>(npts) * static_cast<size_t>(ndims));
  f.read(out.data(), out.size() * sizeof(T), what);
  return out;
}

// pq_search.cu:62-114
PQTables read_pq(const std::string& pivots_file, const std::string& compressed_file) {
  PQTables pq;
  {
    File f(compressed_file);
    int32_t n, m;
    pq.codes = read_bin<uint8_t>(f, 0, n, m, compressed_file);
    pq.num_points = n;
    pq.num_chunks = m;
  }
  File f(pivots_file);
  int32_t nr, nc;
  auto offs = read_bin<uint64_t>(f, 0, nr, nc, pivots_file);
  if (!((nr == 4 || nr == 5) && nc == 1))
    throw IoError(QV_ERR_BAD_INDEX, "PQ pivots metadata must be 4x1 or 5x1 in " + pivots_file);
  const int chunk_idx = (nr == 5) ? 3 : 2;
  int32_t np, dim;
  pq.pivots = read_bin<float>(f, static_cast<int64_t>(offs[0]), np, dim, pivots_file);
  if (np != 256) throw IoError(QV_ERR_BAD_INDEX, "PQ pivots must have 256 rows in " + pivots_file);
  pq.dim = dim;
  int32_t cr, cc;
  pq.centroid = read_bin<float>(f, static_cast<int64_t>(offs[1]), cr, cc, pivots_file);
  if (cr != dim || cc != 1) throw IoError(QV_ERR_BAD_INDEX, "PQ centroid shape mismatch in " + pivots_file);
  pq.chunk_offsets = read_bin<int32_t>(f, static_cast<int64_t>(offs[chunk_idx]), cr, cc, pivots_file);
  if (cr != pq.num_chunks + 1 || cc != 1)
    throw IoError(QV_ERR_BAD_INDEX, "PQ chunk offsets do not match the code width in " + pivots_file);
  return pq;
}

void check_layout(const Layout& L, const PQTables* pq) {
  auto bad = [](const std::string& m) { throw IoError(QV_ERR_BAD_INDEX, m); };
  if (L.num_points <= 0) bad("index holds no points");
  if (L.num_points > 0x7fffffffLL) bad("more than 2^31-1 points is not supported (ids are int32)");
  if (L.max_degree < 1 || L.max_degree > 128) bad("graph degree R must be in [1, 128]");
  if (L.node_size % 4 || L.data_size % 4) bad("node records must be 4-byte aligned (dim * elem % 4 == 0)");
  if (L.nodes_per_page * L.node_size > kPage) bad("nodes_per_page * node_size exceeds a 4 KB page");
  if (L.medoid < 0 || L.medoid >= L.num_points) bad("medoid outside [0, N)");
  if (!pq) return;
  if (pq->dim != L.dim) bad("PQ pivots dimension differs from the index dimension");
  if (pq->num_points != L.num_points) bad("PQ code count differs from the index point count");
  if (pq->num_chunks < 1) bad("PQ code width must be positive");
  const auto& o = pq->chunk_offsets;
  if (o.front() != 0 || o.back() != L.dim) bad("PQ chunk offsets must start at 0 and end at dim");
  for (size_t c = 0; c + 1 < o.size(); ++c)
    if (o[c + 1] < o[c]) bad("PQ chunk offsets must be non-decreasing");
}

// mem_loader.cpp:28-85
void read_pages(const std::string& path, int64_t num_pages, const std::string& backend, uint8_t* dst) {
  const int64_t bytes = num_pages * kPage;
  if (backend == "heap") {
    File f(path);
    f.seek(kPage, path);
    f.read(dst, static_cast<size_t>(bytes), path + " (page store)");
    return;
  }
  if (backend != "mmap") throw IoError(QV_ERR_INVALID_ARG, "memory backend must be heap or mmap");
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw IoError(QV_ERR_IO, "Failed to open mmap Mem Index " + path);
  struct stat st {};
  if (fstat(fd, &st) != 0 || st.st_size < (num_pages + 1) * kPage) {
    ::close(fd);
    throw IoError(QV_ERR_BAD_INDEX, "mmap Mem Index " + path + " is too small");
  }
  void* m = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
  if (m == MAP_FAILED) {
    ::close(fd);
    throw IoError(QV_ERR_IO, "Failed to mmap Mem Index " + path);
  }
  std::memcpy(dst, static_cast<const uint8_t*>(m) + kPage, static_cast<size_t>(bytes));
  munmap(m, static_cast<size_t>(st.st_size));
  ::close(fd);
}

void read_page_range(const std::string& path, int64_t num_pages, const std::string& backend, int64_t first,
                     int64_t count, uint8_t* dst) {
  if (first < 0 || count < 0 || first + count > num_pages)
    throw IoError(QV_ERR_INVALID_ARG, "page range outside the page store");
  if (count == 0) return;
  const size_t bytes = static_cast<size_t>(count) * kPage;
  if (backend == "heap") {
    File f(path);
    f.seek((first + 1) * kPage, path);
    f.read(dst, bytes, path + " (page store)");
    return;
  }
  if (backend != "mmap") throw IoError(QV_ERR_INVALID_ARG, "memory backend must be heap or mmap");
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw IoError(QV_ERR_IO, "Failed to open mmap Mem Index " + path);
  struct stat st {};
  if (fstat(fd, &st) != 0 || st.st_size < (num_pages + 1) * kPage) {
    ::close(fd);
    throw IoError(QV_ERR_BAD_INDEX, "mmap Mem Index " + path + " is too small");
  }
  void* m = mmap(nullptr, bytes, PROT_READ, MAP_PRIVATE, fd, static_cast<off_t>((first + 1) * kPage));
  if (m == MAP_FAILED) {
    ::close(fd);
    throw IoError(QV_ERR_IO, "Failed to mmap Mem Index " + path);
  }
  std::memcpy(dst, m, bytes);
  munmap(m, bytes);
  ::close(fd);
}

void read_stripe_pages(const std::string& path, int64_t num_pages, int32_t num_stripes, int32_t rank,
                       uint8_t* dst) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw IoError(QV_ERR_IO, "Failed to open page file " + path);
  struct stat st {};
  if (fstat(fd, &st) != 0 || st.st_size < (num_pages + 1) * kPage) {
    ::close(fd);
    throw IoError(QV_ERR_BAD_INDEX, "page file " + path + " is too small");
  }
  void* m = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
  if (m == MAP_FAILED) {
    ::close(fd);
    throw IoError(QV_ERR_IO, "Failed to map page file " + path);
  }
  const uint8_t* src = static_cast<const uint8_t*>(m) + kPage;
  int64_t j = 0;
  for (int64_t p = rank; p < num_pages; p += num_stripes, ++j)
    std::memcpy(dst + static_cast<size_t>(j) * kPage, src + static_cast<size_t>(p) * kPage, kPage);
  munmap(m, static_cast<size_t>(st.st_size));
  ::close(fd);
}

int64_t validate_adjacency(const Layout& L, const uint8_t* pages) {
  for (int64_t v = 0; v < L.num_points; ++v) {
    const uint8_t* rec = pages + (v / L.nodes_per_page) * kPage + (v % L.nodes_per_page) * L.node_size;
    uint32_t deg;
    std::memcpy(&deg, rec + L.data_size, 4);
    if (deg > static_cast<uint32_t>(L.max_degree)) return v;
    for (uint32_t t = 0; t < deg; ++t) {
      uint32_t nb;
      std::memcpy(&nb, rec + L.data_size + 4 + 4 * static_cast<int64_t>(t), 4);
      if (static_cast<int64_t>(nb) >= L.num_points) return v;
    }
  }
  return -1;
}

// nav_graph.cu:12-73: nav_index.data = i32 num_node, i32 data_len, vectors;
// map.txt = num_node integers; nav_index = six i32 (field 2 max_m, field 3
// start) then per node i32 degree and that many ids.
NavHost read_nav(const std::string& nav_dir, int64_t elem_size) {
  NavHost nav;
  const std::string data_file = (fs::path(nav_dir) / "nav_index.data").string();
  const std::string map_file = (fs::path(nav_dir) / "map.txt").string();
  const std::string index_file = (fs::path(nav_dir) / "nav_index").string();
  {
    File f(data_file);
    int32_t hdr[2];
    f.read(hdr, sizeof(hdr), data_file);
    nav.num_node = hdr[0];
    nav.data_len = hdr[1];
    if (nav.num_node <= 0 || nav.data_len <= 0)
      throw IoError(QV_ERR_BAD_INDEX, "nav data header: num_node and data_len must be positive");
    nav.data.resize(static_cast<size_t>(nav.num_node) * nav.data_len * elem_size);
    f.read(nav.data.data(), nav.data.size(), data_file);
  }
  {
    std::FILE* f = std::fopen(map_file.c_str(), "r");
    if (!f) throw IoError(QV_ERR_IO, "Failed to open map file: " + map_file);
    nav.mapping.resize(nav.num_node);
    for (int32_t i = 0; i < nav.num_node; ++i) {
      long x = -1;
      if (std::fscanf(f, "%ld", &x) != 1) {
        std::fclose(f);
        throw IoError(QV_ERR_BAD_INDEX, "Failed to read map entry " + std::to_string(i) + " from " + map_file);
      }
      nav.mapping[i] = static_cast<int32_t>(x);
    }
    std::fclose(f);
  }
  {
    File f(index_file);
    int32_t hdr[6];
    f.read(hdr, sizeof(hdr), index_file);
    nav.max_m = hdr[2];
    nav.start = hdr[3];
    if (nav.max_m <= 0 || nav.max_m > 32)
      throw IoError(QV_ERR_BAD_INDEX, "nav_index: max_m must be in (0, 32], got " + std::to_string(nav.max_m));
    nav.graph.assign(static_cast<size_t>(nav.num_node) * nav.max_m, -1);
    for (int32_t i = 0; i < nav.num_node; ++i) {
      int32_t d = 0;
      f.read(&d, 4, index_file);
      if (d <= 0 || d > nav.max_m)
        throw IoError(QV_ERR_BAD_INDEX, "nav_index: node " + std::to_string(i) + " has degree " +
                                            std::to_string(d) + " outside (0, max_m]");
      f.read(nav.graph.data() + static_cast<size_t>(i) * nav.max_m, 4 * static_cast<size_t>(d), index_file);
    }
  }
  return nav;
}

void check_nav(const NavHost& nav, int64_t dim, int64_t num_points) {
  if (nav.num_node <= 0) throw IoError(QV_ERR_BAD_INDEX, "nav graph has no nodes");
  if (nav.max_m <= 0 || nav.max_m > 32) throw IoError(QV_ERR_BAD_INDEX, "nav max_m must be in (0, 32]");
  if (nav.data_len != dim)
    throw IoError(QV_ERR_BAD_INDEX, "nav vectors have " + std::to_string(nav.data_len) + " dims, the index " +
                                        std::to_string(dim));
  if (nav.start < 0 || nav.start >= nav.num_node) throw IoError(QV_ERR_BAD_INDEX, "nav start out of range");
  for (size_t i = 0; i < nav.graph.size(); ++i)
    if (nav.graph[i] < -1 || nav.graph[i] >= nav.num_node)
      throw IoError(QV_ERR_BAD_INDEX, "nav graph id out of range at row " + std::to_string(i / nav.max_m));
  for (int32_t i = 0; i < nav.num_node; ++i)
    if (nav.mapping[i] < 0 || nav.mapping[i] >= num_points)
      throw IoError(QV_ERR_BAD_INDEX, "nav map entry " + std::to_string(i) + " is not a base id");
}

}  // namespace qv
