// expf_table.cpp — the inputs on which this host's libm expf (what rustc's
// f32::exp calls) differs from the correctly rounded binary32 exponential.
//
// The table is built by evaluating both over every binary32 input that can
// produce a finite non-zero result, and is stored as a sorted list of input
// bit patterns. The device exponential (exactmath.h) rounds e^x once from
// double precision and flips to the neighbouring value for listed inputs, so
// device sigmoid and Sinkhorn reproduce the reference's f32::exp exactly.
#include "expf_table.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <mutex>
#include <stdexcept>
#include <thread>
#include <vector>

namespace nbx {

static const char kMagic[8] = {'N', 'B', 'E', 'X', 'P', 'F', '1', '\0'};

ExpfTable scan_expf_exceptions(unsigned threads) {
  ExpConstants C = make_exp_constants();
  if (threads == 0) threads = std::max(1u, std::thread::hardware_concurrency());
  std::vector<std::vector<uint32_t>> found(threads);
  std::atomic<uint64_t> far_mismatches{0};
  std::vector<std::thread> pool;
  const uint64_t total = 1ull << 32;
  for (unsigned t = 0; t < threads; ++t) {
    pool.emplace_back([&, t] {
      uint64_t lo = total * t / threads, hi = total * (t + 1) / threads;
      uint64_t far = 0;
      for (uint64_t u = lo; u < hi; ++u) {
        float x = bits_float((uint32_t)u);
        if (!(x >= -110.0f && x <= 89.0f)) continue;
        double y = 0.0;
        float mine = exp_binary32_host(x, C, &y);
        float libm = std::exp(x);
        if (float_bits(mine) == float_bits(libm)) continue;
        if (near_midpoint(y, mine, C.near_relative) && float_bits(other_neighbour(y, mine)) == float_bits(libm)) {
          found[t].push_back((uint32_t)u);
        } else {
          ++far;
        }
      }
      far_mismatches += far;
    });
  }
  for (auto& th : pool) th.join();
  ExpfTable table;
  for (auto& f : found) table.keys.insert(table.keys.end(), f.begin(), f.end());
  std::sort(table.keys.begin(), table.keys.end());
  table.unexplained = far_mismatches.load();
  return table;
}

void write_expf_table(const char* path, const ExpfTable& table) {
  std::ofstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error(std::string("cannot write ") + path);
  uint32_t count = (uint32_t)table.keys.size();
  f.write(kMagic, 8);
  f.write(reinterpret_cast<const char*>(&count), 4);
  f.write(reinterpret_cast<const char*>(table.keys.data()), (std::streamsize)count * 4);
  if (!f) throw std::runtime_error(std::string("short write to ") + path);
}

bool read_expf_table(const char* path, ExpfTable& table) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  char magic[8];
  uint32_t count = 0;
  f.read(magic, 8);
  f.read(reinterpret_cast<char*>(&count), 4);
  if (!f || std::memcmp(magic, kMagic, 8) != 0 || count > (1u << 24)) return false;
  table.keys.resize(count);
  f.read(reinterpret_cast<char*>(table.keys.data()), (std::streamsize)count * 4);
  return (bool)f;
}

// Spot checks that a loaded table describes this host's expf: every 97th
// listed input, and a spread of unlisted inputs, must round as predicted.
bool verify_expf_table(const ExpfTable& table) {
  ExpConstants C = make_exp_constants();
  for (size_t i = 0; i < table.keys.size(); i += 97) {
    float x = bits_float(table.keys[i]);
    double y = 0.0;
    float mine = exp_binary32_host(x, C, &y);
    if (float_bits(other_neighbour(y, mine)) != float_bits(std::exp(x))) return false;
  }
  uint32_t state = 12345u;
  for (int i = 0; i < 200000; ++i) {
    state = state * 1664525u + 1013904223u;
    float x = bits_float(state);
    if (!(x >= -110.0f && x <= 89.0f)) continue;
    if (std::binary_search(table.keys.begin(), table.keys.end(), state)) continue;
    if (float_bits(exp_binary32_host(x, C)) != float_bits(std::exp(x))) return false;
  }
  return true;
}

std::vector<uint32_t> hash_slots(const ExpfTable& table, uint32_t& mask) {
  uint32_t capacity = 1024;
  while (capacity < table.keys.size() * 3) capacity <<= 1;
  mask = capacity - 1;
  std::vector<uint32_t> slots(capacity, 0u);
  for (uint32_t key : table.keys) {
    uint32_t i = exception_hash(key) & mask;
    while (slots[i] != 0) i = (i + 1) & mask;
    slots[i] = key;
  }
  return slots;
}

}  // namespace nbx
