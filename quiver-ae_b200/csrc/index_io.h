// index_io.h -- DiskANN-layout index files on the host.
//
// Reads the files Quiver's search consumes, with the reference's rules
// (paths inside ruc-system/quiver-ae):
//   *_disk.index header       bin/common/metadata.hpp:15-72
//   *_pq_pivots.bin           src/shared/index/pq_search.cu:62-114 (nr = 4 or 5)
//   *_pq_compressed.bin       src/shared/index/pq_search.cu:67-68
//   page file (header page skipped)  src/shared/io/mem_loader.cpp:28-85
//   index discovery           bin/common/index_discovery.hpp:57-115
//   nav graph                 src/shared/index/nav_graph.cu:12-73
//   query / ground-truth bins bin/common/data_io.hpp:23-133
// Errors are reported as qv::IoError (caught at the C ABI).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace qv {

constexpr int64_t kPage = 4096;

struct IoError : std::runtime_error {
  int code;
  IoError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

struct Layout {
  int64_t num_points = 0, dim = 0, max_degree = 0, node_size = 0, data_size = 0;
  int64_t nodes_per_page = 0, num_pages = 0, medoid = 0;
  int32_t data_type = 0;
};

struct PQTables {
  int32_t dim = 0, num_chunks = 0;
  int64_t num_points = 0;
  std::vector<float> pivots;         // [256 x dim] as stored
  std::vector<float> centroid;       // [dim]
  std::vector<int32_t> chunk_offsets;  // [M + 1]
  std::vector<uint8_t> codes;        // [N x M]
};

int64_t element_size(int32_t data_type);

std::string find_index_file(const std::string& index_dir);
std::string find_pq_prefix(const std::string& index_dir);
std::string find_nav_dir(const std::string& index_dir);

Layout parse_disk_index_header(const std::string& path, int32_t data_type);
PQTables read_pq(const std::string& pivots_file, const std::string& compressed_file);

// Validate geometry the kernels rely on; throws IoError(QV_ERR_BAD_INDEX).
void check_layout(const Layout& L, const PQTables* pq);

// Read pages [1, num_pages] of the index file into `dst` (num_pages * 4096
// bytes).  backend: "heap" (fread) or "mmap" (map then copy).
void read_pages(const std::string& path, int64_t num_pages, const std::string& backend,
                uint8_t* dst);
// Pages [first, first + count) of the page store (page p is file page p + 1),
// with the same backends as read_pages; the file must hold all num_pages.
void read_page_range(const std::string& path, int64_t num_pages, const std::string& backend, int64_t first,
                     int64_t count, uint8_t* dst);
// Pages rank, rank + S, rank + 2S, ... of the page file (one stripe of S),
// gathered through a read-only mapping so only those pages are touched.
void read_stripe_pages(const std::string& path, int64_t num_pages, int32_t num_stripes, int32_t rank,
                       uint8_t* dst);

// Scan every record: degree <= R and neighbour ids < N.  Returns the first
// offending node or -1.
int64_t validate_adjacency(const Layout& L, const uint8_t* pages);

// A navigation graph as NavGraph::init reads it (nav_index, nav_index.data,
// map.txt in one directory).  Rows of `graph` are max_m wide, -1 padded.
struct NavHost {
  int32_t num_node = 0, data_len = 0, max_m = 0, start = 0;
  std::vector<uint8_t> data;      // [num_node x data_len] elements of the base type
  std::vector<int32_t> graph;     // [num_node x max_m]
  std::vector<int32_t> mapping;   // [num_node]
};

NavHost read_nav(const std::string& nav_dir, int64_t elem_size);

// Checks the kernels rely on (the reference asserts some of them and reads
// out of bounds on the rest): 0 < max_m <= 32, start < num_node, data_len ==
// dim, graph ids -1 or < num_node, mapping ids < num_points.  Throws
// IoError(QV_ERR_BAD_INDEX).
void check_nav(const NavHost& nav, int64_t dim, int64_t num_points);

}  // namespace qv
