// CudaExecutor: the B200 counterpart of rocm::ROCmExecutor
// (include/pyflame/backend/rocm/rocm_executor.hpp:37-194).
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/pyflame_cuda.h"
#include "compiler.hpp"
#include "graph.hpp"
#include "memory_pool.hpp"
#include "plan.hpp"

namespace pfb {

// Constants whose elements are all equal (and data-less leaves, which read as
// zero) become scalars: node id -> value.
std::unordered_map<uint64_t, float> detect_splats(const Graph& g, const std::vector<uint64_t>& order,
                                                  const std::unordered_set<uint64_t>& bindings);

class CudaExecutor {
 public:
  explicit CudaExecutor(const pfc_executor_config& cfg);
  ~CudaExecutor();
  CudaExecutor(const CudaExecutor&) = delete;
  CudaExecutor& operator=(const CudaExecutor&) = delete;

  // Host-buffer path (ROCmExecutor::execute, rocm_executor.cpp:66-161).
  void execute(Graph& g, const std::vector<uint64_t>& outs, void* const* host_out, const size_t* out_bytes,
               pfc_execution_result* res);
  // Device-resident path: caller device pointers for inputs and outputs.
  void execute_device(Graph& g, const std::vector<uint64_t>& in_ids, const void* const* in_dev,
                      const std::vector<uint64_t>& outs, void* const* out_dev, cudaStream_t stream,
                      pfc_execution_result* res);
  // Streamed host-buffer path: `g` computes one chunk of rows; the inputs
  // and outputs hold n_chunks chunks back to back.  Copies of chunk c+1 in
  // and c-1 out overlap the compute of chunk c (three streams, two slots).
  void execute_streamed(Graph& g, const std::vector<uint64_t>& in_ids, const void* const* in_host,
                        const std::vector<uint64_t>& outs, void* const* out_host, int n_chunks,
                        pfc_execution_result* res);

  pfc_device_info device_info() const;
  pfc_memory_stats memory_stats() const { return pool_->stats(); }
  cudaError_t release_constants();  // first CUDA error met while releasing
  // Caller-owned device memory holding the payload of constants keyed
  // (cache_key, bytes): used in place of an upload, never written or freed.
  void set_resident(uint64_t cache_key, const void* dev, size_t bytes);
  std::string describe(Graph& g, const std::vector<uint64_t>& outs);
  const std::vector<std::pair<std::string, double>>& last_profile() const { return profile_; }

 private:
  // host->device bytes copied during the current call (resident uploads, per-call
  // constants, inputs, the splat table); reported in pfc_execution_result
  uint64_t h2d_ = 0;
  struct PlanEntry {
    std::unique_ptr<Plan> plan;
    void* arena = nullptr;
    // split-last-wave workspace of the plan's GEMMs (one 128 x 128 fp32 slot
    // per SM, then kTailCounters zeroed counters); null without plain GEMMs.
    // Like the arena, one execution of the plan at a time uses it.
    void* tail = nullptr;
    std::vector<cudaKernel_t> kernels;  // per step (JIT steps)
    // captured CUDA graphs of the plan, one per set of buffer pointers (a
    // streamed call alternates between two sets); at most kGraphsPerPlan
    std::vector<std::pair<std::vector<void*>, cudaGraphExec_t>> graphs;
    int runs = 0;
    std::vector<float> table;           // splat values last uploaded to the scalar table
    void* table_ptr = nullptr;
    // streamed execution: two device slots per streamed input and output,
    // kept with the plan (allocating them per call made the pool trim and
    // re-map memory on every call)
    std::vector<void*> slots[2];
    std::vector<size_t> slot_bytes;
  };
  // The last (graph, version, outputs, bindings) prepared and its plan: a
  // repeated call on an unchanged graph skips validation, the topological
  // walk, splat detection and the structural hash (its per-call splat leaves
  // are re-checked).
  struct LastPrepared {
    uint64_t graph_uid = 0, version = 0;
    std::vector<uint64_t> outs, bindings;
    PlanEntry* pe = nullptr;
  } last_;
  struct Resident {
    void* dev = nullptr;
    size_t bytes = 0;
    bool owned = true;   // false: registered by the caller (set_resident)
  };
  struct Prepared {      // operand derived from a resident constant (BufKind::PREPARED)
    void* dev = nullptr;
    size_t bytes = 0;
    bool filled = false;
  };
  struct SplatInfo {
    bool splat = false;
    float value = 0.f;
  };

  pfc_executor_config cfg_;
  cudaStream_t stream_ = nullptr;
  cudaStream_t copy_in_ = nullptr, copy_out_ = nullptr;  // streamed execution (created on first use)
  std::unique_ptr<CudaMemoryPool> pool_;
  int* err_dev_ = nullptr;
  int num_sms_ = 148;
  static constexpr int kTailCounters = 1024;
  size_t tail_ws_bytes() const { return (size_t)num_sms_ * 128 * 128 * sizeof(float); }
  std::mutex mu_;
  std::unordered_map<uint64_t, PlanEntry> plans_;
  std::map<std::pair<uint64_t, size_t>, Resident> resident_;
  std::map<std::pair<uint64_t, size_t>, SplatInfo> resident_splat_;
  std::unordered_map<uint64_t, Prepared> prepared_;
  std::vector<std::pair<std::string, double>> profile_;

  PlanEntry& prepare(Graph& g, const std::vector<uint64_t>& outs, const std::unordered_set<uint64_t>& bindings,
                     double* compile_ms);
  std::unordered_map<uint64_t, float> detect_splats(const Graph& g, const std::vector<uint64_t>& order,
                                                    const std::unordered_set<uint64_t>& bindings);
  std::vector<void*> resolve(PlanEntry& pe, const Graph& g, const std::unordered_map<uint64_t, const void*>& bind,
                             cudaStream_t s, std::vector<std::pair<void*, const Node*>>* uploads);
  int64_t run_steps(PlanEntry& pe, const std::vector<void*>& ptrs, cudaStream_t s);
  void launch_step(PlanEntry& pe, size_t i, const std::vector<void*>& ptrs, cudaStream_t s);
  void check_device_error(cudaStream_t s);
};

}  // namespace pfb
