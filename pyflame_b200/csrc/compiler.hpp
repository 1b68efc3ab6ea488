// Graph -> Plan compiler: attribute normalisation, strided views for shape
// ops, fusion (elementwise regions, row operations with their elementwise
// prologue, GEMM/conv epilogues), buffer liveness and arena layout, and
// generation of the fused kernels' CUDA source.
#pragma once

#include <memory>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "graph.hpp"
#include "plan.hpp"

namespace pfb {

struct CompileInput {
  const Graph* g = nullptr;
  std::vector<uint64_t> outputs;
  std::unordered_map<uint64_t, float> splats;   // constant node -> value of every element
  std::unordered_set<uint64_t> bindings;         // nodes whose data is a caller device pointer
  int precision = 0;
  int num_sms = 148;
};

// Generated kernel sources of a plan, by module key.
using SourceMap = std::unordered_map<std::string, std::pair<std::string, std::string>>;  // key -> (source, kernel)

std::unique_ptr<Plan> compile_plan(const CompileInput& in, SourceMap* sources);

}  // namespace pfb
