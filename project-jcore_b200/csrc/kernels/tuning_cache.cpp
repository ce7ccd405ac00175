// Persistent tile-configuration cache (see tuning_cache.h).
//
// File format (text, one record per line):
//   npl_b200-tuning-cache <version>
//   hardware <signature>
//   <key>\t<choice>\t<microseconds>\t<unix time>
// Loading checks the version and the hardware signature (device name,
// compute capability, SM count, L2 size), as the reference's cache checks
// CACHE_VERSION and its CPU signature (tuning_cache.cpp LoadBinary), and
// rejects the whole file on a mismatch.
#include "tuning_cache.h"

#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <ctime>
#include <fstream>
#include <mutex>
#include <sstream>
#include <unordered_map>
#include <vector>

#include "nplk_host.h"

namespace nplk {
namespace {

constexpr int kCacheVersion = 1;
constexpr const char *kMagic = "npl_b200-tuning-cache";

struct Entry {
  int choice;
  double us;
  uint64_t stamp;
  uint64_t seq;  // insertion order, for eviction
};

struct Cache {
  std::mutex mu;
  std::unordered_map<std::string, Entry> map;
  std::atomic<size_t> size{0};
  std::atomic<uint64_t> hits{0}, misses{0}, tunes{0}, evictions{0};
  size_t max_entries = 0;  // 0 = unlimited
  uint64_t next_seq = 0;
};

Cache &cache() {
  static Cache c;
  return c;
}

std::string hardware_signature() {
  int dev = 0;
  cudaDeviceProp prop{};
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
    cudaGetLastError();
    return "no-device";
  }
  std::ostringstream os;
  os << prop.name << "|cc=" << prop.major << "." << prop.minor
     << "|sm=" << prop.multiProcessorCount << "|l2=" << prop.l2CacheSize;
  std::string s = os.str();
  for (char &ch : s)
    if (ch == '\t' || ch == '\n') ch = ' ';
  return s;
}

// Inserts with the cache's mutex held.
void insert_locked(Cache &c, const std::string &key, int choice, double us, uint64_t stamp) {
  auto it = c.map.find(key);
  if (it != c.map.end()) {
    it->second = Entry{choice, us, stamp, c.next_seq++};
  } else {
    c.map.emplace(key, Entry{choice, us, stamp, c.next_seq++});
  }
  while (c.max_entries > 0 && c.map.size() > c.max_entries) {
    auto oldest = c.map.begin();
    for (auto e = c.map.begin(); e != c.map.end(); ++e)
      if (e->second.seq < oldest->second.seq) oldest = e;
    c.map.erase(oldest);
    c.evictions++;
  }
  c.size = c.map.size();
}

}  // namespace

std::string tuning_key_conv(const nplk_conv_geom_t *g) {
  std::ostringstream os;
  os << "conv n=" << g->n << " c=" << g->c_in << " h=" << g->h << " w=" << g->w
     << " co=" << g->c_out << " k=" << g->kh << "x" << g->kw << " s=" << g->stride_h << "x"
     << g->stride_w << " p=" << g->pad_top << "x" << g->pad_left << " d=" << g->dil_h << "x"
     << g->dil_w << " o=" << g->h_out << "x" << g->w_out << " sm=" << sm_count();
  return os.str();
}

std::string tuning_key_gemm(int64_t M, int64_t N, int64_t K) {
  std::ostringstream os;
  os << "gemm m=" << M << " n=" << N << " k=" << K << " sm=" << sm_count();
  return os.str();
}

bool tuning_cache_empty() { return cache().size.load(std::memory_order_relaxed) == 0; }

bool tuning_lookup(const std::string &key, int *choice) {
  Cache &c = cache();
  if (c.size.load(std::memory_order_relaxed) == 0) {
    c.misses++;
    return false;
  }
  std::lock_guard<std::mutex> lock(c.mu);
  auto it = c.map.find(key);
  if (it == c.map.end()) {
    c.misses++;
    return false;
  }
  c.hits++;
  *choice = it->second.choice;
  return true;
}

void tuning_insert(const std::string &key, int choice, double us) {
  Cache &c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  insert_locked(c, key, choice, us, static_cast<uint64_t>(std::time(nullptr)));
  c.tunes++;
}

}  // namespace nplk

using namespace nplk;

extern "C" int nplk_tuning_cache_load(const char *path) {
  if (!path) return kErrInvalidArg;
  std::ifstream in(path);
  if (!in) return kErrInvalidArg;
  std::string line, magic;
  int version = 0;
  if (!std::getline(in, line)) return kErrInvalidArg;
  {
    std::istringstream hs(line);
    if (!(hs >> magic >> version) || magic != kMagic) return kErrInvalidArg;
  }
  if (version != kCacheVersion) {
    std::fprintf(stderr, "[NPL] tuning cache %s: version %d, this library reads %d\n", path,
                 version, kCacheVersion);
    return kErrUnsupported;
  }
  if (!std::getline(in, line) || line.rfind("hardware ", 0) != 0) return kErrInvalidArg;
  const std::string hw = line.substr(9);
  if (hw != hardware_signature()) {
    std::fprintf(stderr, "[NPL] tuning cache %s: recorded on '%s', this device is '%s'\n", path,
                 hw.c_str(), hardware_signature().c_str());
    return kErrUnsupported;
  }
  struct Rec {
    std::string key;
    int choice;
    double us;
    uint64_t stamp;
  };
  std::vector<Rec> recs;
  while (std::getline(in, line)) {
    if (line.empty()) continue;
    const size_t t1 = line.find('\t');
    if (t1 == std::string::npos) return kErrInvalidArg;
    Rec r;
    r.key = line.substr(0, t1);
    std::istringstream rs(line.substr(t1 + 1));
    if (!(rs >> r.choice >> r.us >> r.stamp)) return kErrInvalidArg;
    recs.push_back(std::move(r));
  }
  Cache &c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  for (const Rec &r : recs) insert_locked(c, r.key, r.choice, r.us, r.stamp);
  return static_cast<int>(recs.size());
}

extern "C" int nplk_tuning_cache_save(const char *path) {
  if (!path) return kErrInvalidArg;
  Cache &c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  const std::string tmp = std::string(path) + ".tmp";
  {
    std::ofstream out(tmp, std::ios::trunc);
    if (!out) return kErrInternal;
    out << kMagic << " " << kCacheVersion << "\n";
    out << "hardware " << hardware_signature() << "\n";
    for (const auto &kv : c.map)
      out << kv.first << "\t" << kv.second.choice << "\t" << kv.second.us << "\t"
          << kv.second.stamp << "\n";
    if (!out) return kErrInternal;
  }
  if (std::rename(tmp.c_str(), path) != 0) return kErrInternal;
  return static_cast<int>(c.map.size());
}

extern "C" void nplk_tuning_cache_clear(void) {
  Cache &c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  c.map.clear();
  c.size = 0;
  c.hits = 0;
  c.misses = 0;
  c.tunes = 0;
  c.evictions = 0;
}

extern "C" int nplk_tuning_cache_stats(nplk_tuning_stats_t *out) {
  if (!out) return kErrInvalidArg;
  Cache &c = cache();
  out->entries = c.size.load();
  out->hits = c.hits.load();
  out->misses = c.misses.load();
  out->tunes = c.tunes.load();
  out->evictions = c.evictions.load();
  return kOk;
}

extern "C" int nplk_tuning_cache_set_max_entries(size_t n) {
  Cache &c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  c.max_entries = n;
  while (c.max_entries > 0 && c.map.size() > c.max_entries) {
    auto oldest = c.map.begin();
    for (auto e = c.map.begin(); e != c.map.end(); ++e)
      if (e->second.seq < oldest->second.seq) oldest = e;
    c.map.erase(oldest);
    c.evictions++;
  }
  c.size = c.map.size();
  return kOk;
}

namespace {
size_t copy_key(const std::string &k, char *buf, size_t len) {
  if (buf && len > 0) {
    const size_t n = k.size() < len - 1 ? k.size() : len - 1;
    std::memcpy(buf, k.data(), n);
    buf[n] = '\0';
  }
  return k.size();
}
}  // namespace

extern "C" size_t nplk_tuning_key_conv(const nplk_conv_geom_t *g, char *buf, size_t len) {
  if (!g) return 0;
  return copy_key(tuning_key_conv(g), buf, len);
}

extern "C" size_t nplk_tuning_key_gemm(int64_t M, int64_t N, int64_t K, char *buf, size_t len) {
  return copy_key(tuning_key_gemm(M, N, K), buf, len);
}

extern "C" int nplk_tuning_cache_put(const char *key, int choice, float us) {
  if (!key || !key[0] || std::strchr(key, '\t') || std::strchr(key, '\n')) return kErrInvalidArg;
  Cache &c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  insert_locked(c, key, choice, us, static_cast<uint64_t>(std::time(nullptr)));
  return kOk;
}

extern "C" int nplk_tuning_cache_get(const char *key, int *choice, float *us) {
  if (!key) return kErrInvalidArg;
  Cache &c = cache();
  std::lock_guard<std::mutex> lock(c.mu);
  auto it = c.map.find(key);
  if (it == c.map.end()) return 0;
  if (choice) *choice = it->second.choice;
  if (us) *us = static_cast<float>(it->second.us);
  return 1;
}
