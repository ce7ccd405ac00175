// Persistent tile-configuration cache: the kernel choice measured fastest for
// an (operation, shape, SM count) key, kept across runs in a text file.
//
// Counterpart of the reference's tuning result cache
// (composite/tuning_rCache/src/tuning_cache.cpp:186-506, header
// include/tuning_cache.h): a keyed store of tuning outcomes with hit / miss
// statistics, a format version and a hardware signature checked on load, an
// optional entry limit, and explicit save / load / clear. What is tuned here
// is the B200 kernel choice:
//   conv  the implicit-GEMM kernel (NPLK_CONV_ALGO_*), keyed by the full
//         geometry and the SM count;
//   gemm  the output-tile width BN (64 or 128 columns), keyed by M, N, K and
//         the SM count.
// The AUTO paths of nplk_conv2d_run and nplk_gemm consult the cache; the
// nplk_*_tune entry points measure the candidates and fill it. Thread safe.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include "npl_kernels.h"

namespace nplk {

// Canonical keys ("conv n=32 c=64 h=56 w=56 co=64 k=3x3 s=1x1 p=1x1 d=1x1
// o=56x56 sm=148", "gemm m=1024 n=1024 k=1024 sm=148").
std::string tuning_key_conv(const nplk_conv_geom_t *g);
std::string tuning_key_gemm(int64_t M, int64_t N, int64_t K);

// True while the cache holds nothing (a lock-free check that lets callers
// skip building a key).
bool tuning_cache_empty();

// The cached choice for `key` (counts a hit or a miss); false when absent.
bool tuning_lookup(const std::string &key, int *choice);
// Inserts or replaces an entry (evicting the oldest beyond the entry limit).
void tuning_insert(const std::string &key, int choice, double us);

}  // namespace nplk
