// quiver_search -- drop-in replacement for the reference's command-line
// engine (bin/quiver_search.cu), linked against libquiver_b200.so through
// the C ABI in include/quiver_b200.h.
//
// Flags, defaults, validation messages, report lines and result files are
// those of the reference (bin/quiver_search.cu:58-320,
// bin/common/cli_shared.hpp:14-57, bin/common/cli_validation.hpp:9-10,
// bin/common/search_setup.hpp:163-217, src/shared/common/run_report.hpp:96-140),
// so Quiver's Python API (python/quiver/index.py) and the AE log parsers keep
// working.  SPDK-only flags are accepted and ignored; an SSD list is
// rejected as in a build without SPDK.  Added flags: --page-store hbm|host
// (where graph pages live) and --device N.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <map>
#include <numeric>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "quiver_b200.h"

namespace {

struct Args {
  std::string index_dir, query_file, ground_truth_file, data_type, ssd_list_file;
  std::string memory_backend = "heap", memory_index_file, num_blocks_list, result_prefix;
  std::string early_exit_policy = "gpruning", step_recall_csv = "quiver_step_recall.csv", final_recall_csv;
  std::string page_store = "hbm";
  // stream: one persistent launch with the host admitting queries as they
  // complete (the reference's host loop, search.cu:983-1051); batch: every
  // query admitted at the call
  std::string admission = "stream";
  int prefeed = -1, admit_min_batch = 32;
  int topk = 10, ef_search = 30, repeat = 20;
  int num_blocks = 756, poll_threads = 6, pipe_width = 2, queries_per_block = 1, runners_per_ssd = 1;
  int device = 0;
  bool skip_nav = false, per_step_recall = false;
  float recall_threshold = 0.9f;
};

const char* kUsage =
    "Usage: quiver_search --index-dir DIR --query FILE --data-type {uint8,int8,float}\n"
    "  [--topk 10] [--ef-search 30] [--repeat 20] [--ground-truth FILE]\n"
    "  [--memory-backend heap|mmap] [--memory-index-file FILE] [--ssd-list-file FILE]\n"
    "  [--num-blocks 756] [--num-blocks-list LIST] [--queries-per-block 1] [--pipe-width 2]\n"
    "  [--poll-threads 6] [--runners-per-ssd 1] [--early-exit-policy gpruning|none]\n"
    "  [--result-prefix PREFIX] [--final-recall-csv FILE] [--skip-nav]\n"
    "  [--page-store hbm|host] [--device N]\n"
    "  [--admission stream|batch] [--prefeed N] [--admit-min-batch N]\n";

bool parse_int(const std::string& flag, const std::string& v, int& out) {
  try {
    size_t pos = 0;
    out = std::stoi(v, &pos);
    if (pos != v.size()) throw std::invalid_argument(v);
    return true;
  } catch (...) {
    std::cerr << "invalid value for " << flag << ": " << v << std::endl;
    return false;
  }
}

int parse_args(int argc, char** argv, Args& a) {
  // the reference reads these from the environment (search.cu:829-831, 975-977)
  if (const char* v = std::getenv("QUIVER_PREFEED")) a.prefeed = std::atoi(v);
  if (const char* v = std::getenv("QUIVER_ADMIT_MIN_BATCH")) a.admit_min_batch = std::max(1, std::atoi(v));
  std::map<std::string, std::string*> str = {
      {"--index-dir", &a.index_dir}, {"--query", &a.query_file}, {"--ground-truth", &a.ground_truth_file},
      {"--data-type", &a.data_type}, {"--ssd-list-file", &a.ssd_list_file},
      {"--memory-backend", &a.memory_backend}, {"--memory-index-file", &a.memory_index_file},
      {"--num-blocks-list", &a.num_blocks_list}, {"--result-prefix", &a.result_prefix},
      {"--early-exit-policy", &a.early_exit_policy}, {"--step-recall-csv", &a.step_recall_csv},
      {"--final-recall-csv", &a.final_recall_csv}, {"--page-store", &a.page_store},
      {"--admission", &a.admission}};
  std::map<std::string, int*> ints = {
      {"--topk", &a.topk}, {"--ef-search", &a.ef_search}, {"--repeat", &a.repeat},
      {"--num-blocks", &a.num_blocks}, {"--poll-threads", &a.poll_threads}, {"--pipe-width", &a.pipe_width},
      {"--queries-per-block", &a.queries_per_block}, {"--runners-per-ssd", &a.runners_per_ssd},
      {"--device", &a.device}, {"--prefeed", &a.prefeed}, {"--admit-min-batch", &a.admit_min_batch}};
  int ignored = 0;
  std::map<std::string, int*> ignored_ints = {{"--spdk-submit-queue-cap", &ignored},
                                              {"--spdk-task-contexts", &ignored},
                                              {"--spdk-runner-io-contexts", &ignored}};
  for (int i = 1; i < argc; ++i) {
    std::string flag = argv[i], val;
    const auto eq = flag.find('=');
    bool inline_val = false;
    if (eq != std::string::npos) {
      val = flag.substr(eq + 1);
      flag = flag.substr(0, eq);
      inline_val = true;
    }
    if (flag == "--help") {
      std::cout << kUsage;
      std::exit(0);
    }
    if (flag == "--skip-nav") { a.skip_nav = true; continue; }
    if (flag == "--per-step-recall") { a.per_step_recall = true; continue; }
    auto take = [&]() -> bool {
      if (inline_val) return true;
      if (i + 1 >= argc) {
        std::cerr << flag << ": expected a value" << std::endl;
        return false;
      }
      val = argv[++i];
      return true;
    };
    if (auto it = str.find(flag); it != str.end()) {
      if (!take()) return 1;
      *it->second = val;
    } else if (auto jt = ints.find(flag); jt != ints.end()) {
      if (!take() || !parse_int(flag, val, *jt->second)) return 1;
    } else if (auto kt = ignored_ints.find(flag); kt != ignored_ints.end()) {
      if (!take() || !parse_int(flag, val, *kt->second)) return 1;
    } else if (flag == "--recall-threshold") {
      if (!take()) return 1;
      a.recall_threshold = std::strtof(val.c_str(), nullptr);
    } else {
      std::cerr << "Unknown argument: " << flag << std::endl << kUsage;
      return 1;
    }
  }
  if (a.admission != "stream" && a.admission != "batch") {
    std::cerr << "--admission must be stream or batch" << std::endl;
    return 1;
  }
  for (auto req : {std::make_pair("--index-dir", &a.index_dir), std::make_pair("--query", &a.query_file),
                   std::make_pair("--data-type", &a.data_type)}) {
    if (req.second->empty()) {
      std::cerr << req.first << ": required." << std::endl << kUsage;
      return 1;
    }
  }
  return 0;
}

// bin/common/data_io.hpp:23-49
template <class T>
std::vector<T> read_typed_bin(const std::string& path, size_t& dims, size_t& count) {
  std::ifstream in(path, std::ios::binary);
  if (!in) {
    std::cerr << "Failed to open file " << path << std::endl;
    std::exit(1);
  }
  int32_t n = 0, d = 0;
  in.read(reinterpret_cast<char*>(&n), 4);
  in.read(reinterpret_cast<char*>(&d), 4);
  // The reference reads on regardless; a short or malformed file would leave the search
  // uninitialised queries, so it is refused here.
  if (!in || n < 0 || d < 0) {
    std::cerr << "Invalid header in file " << path << std::endl;
    std::exit(1);
  }
  dims = static_cast<size_t>(d);
  count = static_cast<size_t>(n);
  std::vector<T> out(dims * count);
  const auto want = static_cast<std::streamsize>(sizeof(T) * out.size());
  in.read(reinterpret_cast<char*>(out.data()), want);
  if (in.gcount() != want) {
    std::cerr << "File " << path << " is truncated: " << count << " x " << dims << " values expected"
              << std::endl;
    std::exit(1);
  }
  return out;
}

// bin/common/data_io.hpp:73-108
std::vector<float> load_queries_as_float(const std::string& path, int repeat, size_t& dims, size_t& count) {
  std::vector<float> q;
  if (path.find(".u8bin") != std::string::npos) {
    auto raw = read_typed_bin<uint8_t>(path, dims, count);
    q.assign(raw.begin(), raw.end());
  } else if (path.find(".i8bin") != std::string::npos) {
    auto raw = read_typed_bin<int8_t>(path, dims, count);
    q.assign(raw.begin(), raw.end());
  } else {
    q = read_typed_bin<float>(path, dims, count);
  }
  if (repeat > 1) {
    std::vector<float> r(q.size() * repeat);
    for (int i = 0; i < repeat; ++i) std::copy(q.begin(), q.end(), r.begin() + i * q.size());
    q.swap(r);
    count *= static_cast<size_t>(repeat);
  }
  return q;
}

// bin/common/recall.hpp:6-62
struct QueryRecall {
  int hits = 0;
  double recall = 0.0;
};
QueryRecall one_query_recall(const int* res, const int* gt, int topk) {
  QueryRecall r;
  std::set<int> expected(gt, gt + topk);
  for (int j = 0; j < topk; ++j)
    if (expected.count(res[j])) ++r.hits;
  r.recall = static_cast<double>(r.hits) / topk;
  return r;
}
double calc_recall(const int* res, const int* gt, size_t nq, size_t width, int topk) {
  size_t hits = 0;
  for (size_t i = 0; i < nq; ++i) hits += one_query_recall(res + i * topk, gt + i * width, topk).hits;
  return static_cast<double>(hits) / static_cast<double>(nq * topk);
}

// bin/common/data_io.hpp:111-140
template <class T>
void write_typed_bin(const std::string& path, const T* v, size_t count, size_t dims) {
  std::ofstream out(path, std::ios::binary | std::ios::trunc);
  if (!out) throw std::runtime_error("Failed to open binary result file " + path);
  const int32_t c = static_cast<int32_t>(count), d = static_cast<int32_t>(dims);
  out.write(reinterpret_cast<const char*>(&c), 4);
  out.write(reinterpret_cast<const char*>(&d), 4);
  out.write(reinterpret_cast<const char*>(v), static_cast<std::streamsize>(sizeof(T) * count * dims));
  if (!out) throw std::runtime_error("Failed to write binary result file " + path);
}

std::vector<int> parse_int_list(const std::string& raw, const char* name) {
  std::string s = raw;
  std::replace(s.begin(), s.end(), ',', ' ');
  std::istringstream iss(s);
  std::vector<int> v;
  std::string tok;
  while (iss >> tok) {
    try {
      v.push_back(std::stoi(tok));
    } catch (...) {
      std::cerr << "invalid integer in " << name << ": " << tok << std::endl;
      std::exit(1);
    }
  }
  if (v.empty()) {
    std::cerr << "empty list for " << name << std::endl;
    std::exit(1);
  }
  return v;
}

bool ssd_list_nonempty(const std::string& path) {
  if (path.empty()) return false;
  std::ifstream in(path);
  if (!in) {
    std::cerr << "Failed to open SSD list file " << path << std::endl;
    std::exit(1);
  }
  std::string line;
  while (in >> line)
    if (!line.empty()) return true;
  return false;
}

double pct(const std::vector<double>& sorted, double frac) {
  if (sorted.empty()) return 0.0;
  size_t i = static_cast<size_t>(static_cast<double>(sorted.size()) * frac);
  return sorted[std::min(i, sorted.size() - 1)];
}

}  // namespace

int main(int argc, char** argv) {
  Args a;
  if (int rc = parse_args(argc, argv, a)) return rc;
  if (ssd_list_nonempty(a.ssd_list_file)) {
    std::cerr << "This binary was built without SPDK support" << std::endl;
    return 1;
  }
  auto positive = [](int v, const char* n) {
    if (v > 0) return true;
    std::cerr << n << " must be positive" << std::endl;
    return false;
  };
  auto range = [](int v, const char* n, int lo, int hi) {
    if (v >= lo && v <= hi) return true;
    std::cerr << n << " must be in [" << lo << ", " << hi << "]" << std::endl;
    return false;
  };
  if (!positive(a.num_blocks, "--num-blocks") || !positive(a.poll_threads, "--poll-threads") ||
      !range(a.pipe_width, "--pipe-width", 1, 16) ||
      !range(a.queries_per_block, "--queries-per-block", 1, 8))
    return 1;
  int policy;
  if (a.early_exit_policy == "none") {
    policy = QV_EXIT_NONE;
  } else if (a.early_exit_policy == "gpruning") {
    policy = QV_EXIT_GPRUNING;
  } else {
    std::cerr << "invalid --early-exit-policy: " << a.early_exit_policy << " (expected gpruning or none)"
              << std::endl;
    return 1;
  }
  std::cout << "[Quiver] early-exit policy=" << (policy == QV_EXIT_NONE ? "none" : "gpruning") << std::endl;
  if (a.per_step_recall) {
    std::cerr << "--per-step-recall is not supported by the B200 engine" << std::endl;
    return 1;
  }
  const std::vector<int> run_blocks =
      a.num_blocks_list.empty() ? std::vector<int>{a.num_blocks} : parse_int_list(a.num_blocks_list, "--num-blocks-list");
  for (int v : run_blocks)
    if (v <= 0) {
      std::cerr << "--num-blocks-list values must be positive: " << v << std::endl;
      return 1;
    }
  if (!a.result_prefix.empty() && run_blocks.size() != 1) {
    std::cerr << "--result-prefix cannot be combined with a multi-value --num-blocks-list" << std::endl;
    return 1;
  }
  int32_t dtype;
  if (a.data_type == "uint8") dtype = QV_UINT8;
  else if (a.data_type == "float") dtype = QV_FLOAT;
  else if (a.data_type == "int8") dtype = QV_INT8;
  else {
    std::cerr << "Unsupported data type '" << a.data_type << "'. Expected one of: uint8, int8, float" << std::endl;
    return 1;
  }
  if (a.memory_backend != "heap" && a.memory_backend != "mmap") {
    std::cerr << "Unsupported --memory-backend '" << a.memory_backend << "'. Expected one of: heap, mmap"
              << std::endl;
    return 1;
  }
  if (a.page_store != "hbm" && a.page_store != "host") {
    std::cerr << "--page-store must be hbm or host" << std::endl;
    return 1;
  }

  qv_engine_opts eo{};
  eo.index_dir = a.index_dir.c_str();
  eo.data_type = dtype;
  eo.memory_backend = a.memory_backend.c_str();
  eo.memory_index_file = a.memory_index_file.empty() ? nullptr : a.memory_index_file.c_str();
  eo.device = a.device;
  eo.page_store = a.page_store == "host" ? QV_PAGES_HOST : QV_PAGES_HBM;
  qv_engine* eng = nullptr;
  if (qv_engine_create(&eo, &eng) != QV_OK) {
    std::cerr << qv_last_error() << std::endl;
    return 1;
  }
  qv_index_info info{};
  qv_engine_info(eng, &info);
  {
    int32_t nav_nodes = 0, nav_m = 0, nav_start = 0;
    qv_engine_nav_info(eng, &nav_nodes, &nav_m, &nav_start);
    if (nav_nodes > 0)
      std::cout << "[Quiver] NavGraph loaded: " << nav_nodes << " nodes, max_m=" << nav_m << ", start=" << nav_start
                << std::endl;
    else
      std::cout << "[Quiver] No nav_index found in " << a.index_dir << ", skipping NavGraph" << std::endl;
  }

  size_t dims = 0, nq = 0;
  std::vector<float> queries = load_queries_as_float(a.query_file, a.repeat, dims, nq);
  if (dims != static_cast<size_t>(info.dim)) {
    std::cerr << "Query dimension mismatch: query file '" << a.query_file << "' has " << dims
              << " dims, but index '" << a.index_dir << "' expects " << info.dim << " dims" << std::endl;
    qv_engine_destroy(eng);
    return 1;
  }
  if (a.skip_nav)
    std::cout << "[Quiver] --skip-nav enabled: nav graph disabled; all queries start from global enter_point="
              << info.medoid << std::endl;

  std::vector<int32_t> ids(nq * a.topk), found(nq);
  std::vector<float> dists(nq * a.topk), lat(nq);
  for (int nb : run_blocks) {
    if (run_blocks.size() > 1)
      std::cout << "\n============================================================\nQuiver Sweep: num_blocks=" << nb
                << " pipe_width=" << a.pipe_width << " queries_per_block=" << a.queries_per_block
                << "\n============================================================\n" << std::endl;
    qv_search_opts so;
    qv_search_opts_default(&so);
    so.topk = a.topk;
    so.ef_search = a.ef_search;
    so.pipe_width = a.pipe_width;
    so.queries_per_block = a.queries_per_block;
    so.num_blocks = nb;
    so.early_exit_policy = policy;
    so.skip_nav = a.skip_nav ? 1 : 0;
    qv_search_stats plan{};
    if (qv_plan(eng, &so, static_cast<int64_t>(nq), &plan) != QV_OK) {
      std::cerr << qv_last_error() << std::endl;
      qv_engine_destroy(eng);
      return 1;
    }
    double qps = 0, avg = 0, p50 = 0, p90 = 0, p99 = 0, p999 = 0, lmax = 0;
    int64_t expansions = 0;
    std::string admission_params;
    if (a.admission == "stream") {
      qv_stream_opts sto;
      qv_stream_opts_default(&sto);
      sto.prefeed = a.prefeed;
      sto.admit_min_batch = std::max(1, a.admit_min_batch);
      qv_stream_stats ss{};
      if (qv_search_stream(eng, queries.data(), static_cast<int64_t>(nq), info.dim, &so, &sto, ids.data(),
                           dists.data(), found.data(), nullptr, &ss) != QV_OK) {
        std::cerr << qv_last_error() << std::endl;
        qv_engine_destroy(eng);
        return 1;
      }
      qps = ss.qps;
      avg = ss.lat_avg_ms;
      p50 = ss.lat_p50_ms;
      p90 = ss.lat_p90_ms;
      p99 = ss.lat_p99_ms;
      p999 = ss.lat_p999_ms;
      lmax = ss.lat_max_ms;
      expansions = ss.expansions;
      admission_params = " max_inflight=" + std::to_string(ss.max_inflight) +
                         " prefeed=" + std::to_string(ss.max_inflight - ss.workers) +
                         " admissions=" + std::to_string(ss.admissions);
    } else {
      qv_search_stats st{};
      const auto t0 = std::chrono::steady_clock::now();
      if (qv_search_timed(eng, queries.data(), static_cast<int64_t>(nq), info.dim, &so, ids.data(), dists.data(),
                          found.data(), lat.data(), &st) != QV_OK) {
        std::cerr << qv_last_error() << std::endl;
        qv_engine_destroy(eng);
        return 1;
      }
      const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      std::vector<double> l(lat.begin(), lat.end());
      std::sort(l.begin(), l.end());
      qps = secs > 0 ? nq / secs : 0.0;
      avg = l.empty() ? 0.0 : std::accumulate(l.begin(), l.end(), 0.0) / l.size();
      p50 = pct(l, 0.50);
      p90 = pct(l, 0.90);
      p99 = pct(l, 0.99);
      p999 = pct(l, 0.999);
      lmax = l.empty() ? 0.0 : l.back();
      expansions = st.expansions;
    }
    // run_report.hpp:96-140 layout
    std::ostringstream os;
    os << std::fixed;
    os << "========== Quiver Result ==========\n";
    os << "Query Params:\n  topk=" << a.topk << " ef_search=" << a.ef_search << " repeat=" << a.repeat
       << " data_type=" << a.data_type << "\n";
    os << "Runtime Params:\n  num_blocks=" << plan.grid << " pipe_width=" << a.pipe_width
       << " queries_per_block=" << plan.slots_per_block << " task_slots=" << plan.grid * plan.slots_per_block
       << " io_slots=" << plan.grid * plan.slots_per_block * a.pipe_width << " admission=" << a.admission
       << admission_params << " page_store=" << a.page_store << " engine=" << qv_version() << "\n\n";
    os << "Performance:\n  QPS: " << std::setprecision(2) << qps << "\n";
    os << "  QueryLatency(ms): avg=" << std::setprecision(3) << avg << " p50=" << p50 << " p90=" << p90
       << " p99=" << p99 << " p99.9=" << p999 << " max=" << lmax << "\n";
    os << "  SSD Avg Bandwidth: 0.00 GB/s\n  SSD Avg IOPS: 0\n";
    os << "===================================\n";
    std::printf("%s", os.str().c_str());
    std::cout << "[Quiver] Finish summary: policy=" << (policy == QV_EXIT_NONE ? "none" : "gpruning")
              << " avg_finish_step=" << std::fixed << std::setprecision(2)
              << (nq ? static_cast<double>(expansions) / nq : 0.0) << " finished=" << nq << "/" << nq
              << std::defaultfloat << std::endl;

    if (!a.ground_truth_file.empty()) {  // search_setup.hpp:163-174
      size_t gw = 0, gc = 0;
      auto gt = read_typed_bin<int>(a.ground_truth_file, gw, gc);
      const size_t n_eval = std::min(gc, nq);
      std::printf("Recall @ %d: %lf\n", a.topk, calc_recall(ids.data(), gt.data(), n_eval, gw, a.topk));
      if (!a.final_recall_csv.empty()) {  // search_setup.hpp:176-200
        std::ofstream out(a.final_recall_csv);
        out << "query_id,gt_query_id,hits,recall\n";
        for (size_t i = 0; i < nq; ++i) {
          const size_t g = i % gc;
          const auto r = one_query_recall(ids.data() + i * a.topk, gt.data() + g * gw, a.topk);
          out << i << "," << g << "," << r.hits << "," << std::fixed << std::setprecision(6) << r.recall << "\n";
        }
        std::cout << "[Quiver] Per-query recall CSV: " << a.final_recall_csv << std::endl;
      }
    }
    if (!a.result_prefix.empty()) {  // search_setup.hpp:202-217
      try {
        write_typed_bin(a.result_prefix + "_ids.bin", ids.data(), nq, a.topk);
        write_typed_bin(a.result_prefix + "_distances.bin", dists.data(), nq, a.topk);
      } catch (const std::exception& e) {
        std::cerr << e.what() << std::endl;
        qv_engine_destroy(eng);
        return 1;
      }
      std::cout << "[Quiver] Search results: " << a.result_prefix << "_ids.bin " << a.result_prefix
                << "_distances.bin" << std::endl;
    }
  }
  qv_engine_destroy(eng);
  return 0;
}
