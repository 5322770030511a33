// expf_table.h — host side of the libm-compatible device exponential.
#pragma once

#include <cstdint>
#include <vector>

#include "exactmath.h"

namespace nbx {

struct ExpfTable {
  std::vector<uint32_t> keys;  // sorted binary32 input bit patterns
  uint64_t unexplained = 0;    // mismatches the near-midpoint band did not explain (must be 0)
};

ExpfTable scan_expf_exceptions(unsigned threads);
void write_expf_table(const char* path, const ExpfTable& table);
bool read_expf_table(const char* path, ExpfTable& table);
bool verify_expf_table(const ExpfTable& table);
std::vector<uint32_t> hash_slots(const ExpfTable& table, uint32_t& mask);

}  // namespace nbx
