#include "executor.hpp"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <thread>

#include "jit.hpp"
#include "kernels/kernels.hpp"

namespace pfb {

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) PFB_CUDA(cudaSetDevice(dev));
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

double ms_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

// True when every element equals the first (bitwise).  Large buffers are
// scanned by several threads; a mismatch stops all of them.
bool all_equal_f32(const float* p, int64_t n, float* value) {
  uint32_t first;
  std::memcpy(&first, p, 4);
  *value = p[0];
  const uint32_t* u = (const uint32_t*)p;
  auto scan = [&](int64_t b, int64_t e, std::atomic<bool>* stop) {
    for (int64_t i = b; i < e; i += 4096) {
      if (stop->load(std::memory_order_relaxed)) return;
      int64_t end = std::min(e, i + 4096);
      for (int64_t j = i; j < end; ++j)
        if (u[j] != first) {
          stop->store(true);
          return;
        }
    }
  };
  std::atomic<bool> stop{false};
  if (n < (1 << 22)) {
    scan(0, n, &stop);
  } else {
    int nt = (int)std::min<unsigned>(8, std::max(1u, std::thread::hardware_concurrency()));
    std::vector<std::thread> th;
    int64_t chunk = (n + nt - 1) / nt;
    for (int t = 0; t < nt; ++t) {
      int64_t b = t * chunk, e = std::min(n, b + chunk);
      if (b < e) th.emplace_back(scan, b, e, &stop);
    }
    for (auto& t : th) t.join();
  }
  return !stop.load();
}

inline uint64_t mix(uint64_t h, uint64_t v) {
  h ^= v + 0x9e3779b97f4a7c15ULL + (h << 6) + (h >> 2);
  return h * 0xff51afd7ed558ccdULL;
}

}  // namespace

CudaExecutor::CudaExecutor(const pfc_executor_config& cfg) : cfg_(cfg) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) {
    cudaGetLastError();
    fail(PFC_ERR_NO_DEVICE, "CUDA backend requested but no CUDA device is available");
  }
  if (cfg.device_id < 0 || cfg.device_id >= n)
    fail(PFC_ERR_INVALID_ARGUMENT, "device_id " + std::to_string(cfg.device_id) + " out of range (" +
                                       std::to_string(n) + " devices)");
  DeviceGuard dg(cfg.device_id);
  cudaDeviceProp prop;
  PFB_CUDA(cudaGetDeviceProperties(&prop, cfg.device_id));
  if (prop.major < 10)
    fail(PFC_ERR_NO_DEVICE, std::string("device ") + prop.name + " is not sm_100 class (compute capability " +
                                std::to_string(prop.major) + "." + std::to_string(prop.minor) + ")");
  num_sms_ = prop.multiProcessorCount;
  PFB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  CudaMemoryPool::Config pc;
  pc.device = cfg.device_id;
  pc.release_threshold = (cfg.workspace_size_mb ? cfg.workspace_size_mb : 256) << 20;
  pc.fail_after_n = cfg.fail_after_n_allocations;
  pool_ = std::make_unique<CudaMemoryPool>(pc);
  PFB_CUDA(cudaMalloc((void**)&err_dev_, 256));
  PFB_CUDA(cudaMemset(err_dev_, 0, 256));
}

CudaExecutor::~CudaExecutor() {
  DeviceGuard dg(cfg_.device_id);
  if (stream_) cudaStreamSynchronize(stream_);
  (void)release_constants();  // nothing to report to from a destructor
  if (err_dev_) cudaFree(err_dev_);
  pool_.reset();
  if (copy_in_) cudaStreamDestroy(copy_in_);
  if (copy_out_) cudaStreamDestroy(copy_out_);
  if (stream_) cudaStreamDestroy(stream_);
}

cudaError_t CudaExecutor::release_constants() {
  // everything is released even after a failure; the first error is returned
  cudaError_t first = cudaSuccess;
  auto note = [&first](cudaError_t e) {
    if (first == cudaSuccess && e != cudaSuccess) first = e;
  };
  if (stream_) note(cudaStreamSynchronize(stream_));
  for (auto& [k, pe] : plans_) {
    for (auto& gr : pe.graphs) note(cudaGraphExecDestroy(gr.second));
    if (pe.arena) note(pool_->deallocate(pe.arena, stream_));
    if (pe.tail) note(pool_->deallocate(pe.tail, stream_));
    for (int k2 = 0; k2 < 2; ++k2)
      for (void* p : pe.slots[k2]) note(pool_->deallocate(p, stream_));
  }
  plans_.clear();
  last_ = LastPrepared();
  for (auto& [k, r] : resident_) {
    if (!r.owned) continue;
    note(pool_->deallocate(r.dev, stream_));
    pool_->add_resident(-(long long)r.bytes);
  }
  resident_.clear();
  resident_splat_.clear();
  for (auto& [k, pr] : prepared_) {
    note(pool_->deallocate(pr.dev, stream_));
    pool_->add_resident(-(long long)pr.bytes);
  }
  prepared_.clear();
  if (stream_) note(cudaStreamSynchronize(stream_));
  return first;
}

void CudaExecutor::set_resident(uint64_t cache_key, const void* dev, size_t bytes) {
  std::lock_guard<std::mutex> lock(mu_);
  DeviceGuard dg(cfg_.device_id);
  if (!dev || bytes == 0) fail(PFC_ERR_INVALID_ARGUMENT, "set_resident: null pointer or empty payload");
  if (((uintptr_t)dev & 15) != 0) fail(PFC_ERR_INVALID_ARGUMENT, "set_resident: device pointer must be 16-byte aligned");
  auto key = std::make_pair(cache_key, bytes);
  auto it = resident_.find(key);
  if (it != resident_.end() && it->second.owned) {
    if (stream_) PFB_CUDA(cudaStreamSynchronize(stream_));
    PFB_CUDA(pool_->deallocate(it->second.dev, stream_));
    pool_->add_resident(-(long long)it->second.bytes);
  }
  Resident r;
  r.dev = const_cast<void*>(dev);
  r.bytes = bytes;
  r.owned = false;
  resident_[key] = r;
  // operands derived from earlier contents of this key are refilled on next use
  for (auto& [k, pr] : prepared_) pr.filled = false;
}

pfc_device_info CudaExecutor::device_info() const {
  pfc_device_info info;
  std::memset(&info, 0, sizeof info);
  pfc_cuda_get_device_info(cfg_.device_id, &info);
  return info;
}

std::unordered_map<uint64_t, float> detect_splats(const Graph& g, const std::vector<uint64_t>& order,
                                                  const std::unordered_set<uint64_t>& bindings) {
  std::unordered_map<uint64_t, float> out;
  for (uint64_t id : order) {
    const Node& n = g.at(id);
    if (n.type == NodeType::OPERATION || bindings.count(id)) continue;
    if (!n.has_data()) {
      if (n.dtype != DType::F32)
        fail(PFC_ERR_UNSUPPORTED, "node " + std::to_string(id) + " has no data and is not float32");
      out[id] = 0.f;
      continue;
    }
    if (n.dtype != DType::F32 || n.numel() == 0) continue;
    float v = 0.f;
    if (all_equal_f32((const float*)n.data, n.numel(), &v)) out[id] = v;
  }
  return out;
}

std::unordered_map<uint64_t, float> CudaExecutor::detect_splats(const Graph& g, const std::vector<uint64_t>& order,
                                                                const std::unordered_set<uint64_t>& bindings) {
  std::unordered_map<uint64_t, float> out;
  for (uint64_t id : order) {
    const Node& n = g.at(id);
    if (n.type == NodeType::OPERATION || bindings.count(id)) continue;
    if (!n.has_data()) {
      // data-less leaf: zero-filled like the ROCm executor (rocm_executor.cpp:99-102)
      if (n.dtype != DType::F32)
        fail(PFC_ERR_UNSUPPORTED, "node " + std::to_string(id) + " has no data and is not float32");
      out[id] = 0.f;
      continue;
    }
    if (n.data_bytes != n.size_bytes())
      fail(PFC_ERR_INVALID_ARGUMENT, "constant payload of node " + std::to_string(id) + " has " +
                                         std::to_string(n.data_bytes) + " bytes, expected " +
                                         std::to_string(n.size_bytes()));
    if (n.dtype != DType::F32 || n.numel() == 0) continue;
    float v = 0.f;
    bool splat;
    if (n.data_flags & PFC_CONST_RESIDENT) {
      auto key = std::make_pair(n.data_key, n.data_bytes);
      auto it = resident_splat_.find(key);
      if (it == resident_splat_.end()) {
        SplatInfo si;
        si.splat = all_equal_f32((const float*)n.data, n.numel(), &si.value);
        it = resident_splat_.emplace(key, si).first;
      }
      splat = it->second.splat;
      v = it->second.value;
    } else {
      splat = all_equal_f32((const float*)n.data, n.numel(), &v);
    }
    if (splat) out[id] = v;
  }
  return out;
}

CudaExecutor::PlanEntry& CudaExecutor::prepare(Graph& g, const std::vector<uint64_t>& outs,
                                               const std::unordered_set<uint64_t>& bindings, double* compile_ms) {
  auto t0 = std::chrono::steady_clock::now();
  std::vector<uint64_t> bsorted(bindings.begin(), bindings.end());
  std::sort(bsorted.begin(), bsorted.end());
  if (last_.pe && last_.graph_uid == g.uid && last_.version == g.version && last_.outs == outs &&
      last_.bindings == bsorted) {
    // same graph, unchanged: only per-call payloads can differ.  A splat leaf
    // whose payload is per call (not resident) must still hold equal values.
    bool same = true;
    for (auto& sc : last_.pe->plan->scalars) {
      const Node& n = g.at(sc.node);
      if (!n.has_data() || (n.data_flags & PFC_CONST_RESIDENT)) continue;
      float v = 0.f;
      if (!all_equal_f32((const float*)n.data, n.numel(), &v)) {
        same = false;
        break;
      }
      sc.value = v;
    }
    if (same) {
      if (compile_ms) *compile_ms = ms_since(t0);
      return *last_.pe;
    }
  }
  validate_graph(g);
  std::vector<uint64_t> order = topo_order(g, outs);
  auto splats = detect_splats(g, order, bindings);
  uint64_t key = structural_hash(g, outs);
  key = mix(key, (uint64_t)cfg_.precision);
  for (uint64_t x : bsorted) key = mix(key, x ^ 0xb1b1);
  std::vector<uint64_t> sp;
  for (auto& [id, v] : splats) sp.push_back(id);
  std::sort(sp.begin(), sp.end());
  for (uint64_t x : sp) key = mix(key, x ^ 0x5a5a);
  auto it = plans_.find(key);
  if (it == plans_.end()) {
    CompileInput ci;
    ci.g = &g;
    ci.outputs = outs;
    ci.splats = splats;
    ci.bindings = bindings;
    ci.precision = cfg_.precision;
    ci.num_sms = num_sms_;
    SourceMap sources;
    PlanEntry pe;
    pe.plan = compile_plan(ci, &sources);
    pe.plan->key = key;
    pe.kernels.resize(pe.plan->steps.size(), nullptr);
    for (size_t i = 0; i < pe.plan->steps.size(); ++i) {
      Step& s = pe.plan->steps[i];
      if (s.kind != StepKind::JIT) continue;
      const auto& src = sources.at(s.jit.module_key);
      cudaKernel_t k = global_jit().get(s.jit.module_key, src.first, s.jit.kernel);
      pe.kernels[i] = k;
      if (s.jit.smem > 48 * 1024)
        PFB_CUDA(cudaKernelSetAttributeForDevice(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s.jit.smem,
                                                 cfg_.device_id));
      // every generated kernel strides over its work: launch exactly the CTAs
      // that fit on the device at once (no partial second wave)
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, (const void*)k, s.jit.block, s.jit.smem) ==
              cudaSuccess &&
          per_sm > 0) {
        s.jit.grid = std::max(1, std::min(s.jit.grid, per_sm * num_sms_));
      } else {
        cudaGetLastError();
      }
    }
    if (pe.plan->arena_bytes) pe.arena = pool_->allocate(pe.plan->arena_bytes, stream_);
    bool has_gemm = false;
    for (const Step& st : pe.plan->steps) has_gemm = has_gemm || (st.kind == StepKind::GEMM && !st.gemm.conv);
    if (has_gemm) {
      pe.tail = pool_->allocate(tail_ws_bytes() + kTailCounters * sizeof(unsigned), stream_);
      PFB_CUDA(cudaMemsetAsync((char*)pe.tail + tail_ws_bytes(), 0, kTailCounters * sizeof(unsigned), stream_));
    }
    it = plans_.emplace(key, std::move(pe)).first;
  } else {
    // refresh the splat values seen by this call (the structure is unchanged)
    for (auto& sc : it->second.plan->scalars) sc.value = splats.at(sc.node);
  }
  last_.graph_uid = g.uid;
  last_.version = g.version;
  last_.outs = outs;
  last_.bindings = bsorted;
  last_.pe = &it->second;
  if (compile_ms) *compile_ms = ms_since(t0);
  return it->second;
}

std::vector<void*> CudaExecutor::resolve(PlanEntry& pe, const Graph& g,
                                         const std::unordered_map<uint64_t, const void*>& bind, cudaStream_t s,
                                         std::vector<std::pair<void*, const Node*>>* uploads) {
  const Plan& P = *pe.plan;
  std::vector<void*> ptrs(P.buffers.size(), nullptr);
  for (size_t i = 0; i < P.buffers.size(); ++i) {
    const Buffer& b = P.buffers[i];
    switch (b.kind) {
      case BufKind::ARENA:
        if (b.arena_offset >= 0) ptrs[i] = (char*)pe.arena + b.arena_offset;
        break;
      case BufKind::BINDING:
        ptrs[i] = const_cast<void*>(bind.at(b.node));
        break;
      case BufKind::CONST: {
        const Node& n = g.at(b.node);
        if (n.data_flags & PFC_CONST_RESIDENT) {
          auto key = std::make_pair(n.data_key, n.data_bytes);
          auto it = resident_.find(key);
          if (it == resident_.end()) {
            Resident r;
            r.bytes = n.data_bytes;
            r.dev = pool_->allocate(n.data_bytes, s);
            PFB_CUDA(cudaMemcpyAsync(r.dev, n.data, n.data_bytes, cudaMemcpyHostToDevice, s));
            h2d_ += n.data_bytes;
            pool_->add_resident((long long)r.bytes);
            it = resident_.emplace(key, r).first;
          }
          ptrs[i] = it->second.dev;
        } else {
          ptrs[i] = (char*)pe.arena + b.arena_offset;
          uploads->push_back({ptrs[i], &n});
        }
        break;
      }
      case BufKind::PREPARED: {
        auto it = prepared_.find(b.prep_key);
        if (it == prepared_.end()) {
          Prepared pr;
          pr.bytes = b.bytes;
          pr.dev = pool_->allocate(b.bytes, s);
          pool_->add_resident((long long)b.bytes);
          it = prepared_.emplace(b.prep_key, pr).first;
        }
        ptrs[i] = it->second.dev;
        break;
      }
    }
  }
  return ptrs;
}

void CudaExecutor::launch_step(PlanEntry& pe, size_t i, const std::vector<void*>& ptrs, cudaStream_t s) {
  const Plan& P = *pe.plan;
  const Step& st = P.steps[i];
  auto bufp = [&](int buf, int64_t byte_off) -> void* {
    if (buf == kErrorFlagBuffer) return err_dev_;
    if (buf < 0) return nullptr;
    return (char*)ptrs[buf] + byte_off;
  };
  auto viewp = [&](const View& v) -> const float* {
    if (v.is_splat) return (const float*)bufp(P.scalar_buf, (int64_t)v.splat_slot * 4);
    return (const float*)bufp(v.buf, v.offset * (int64_t)dtype_size(v.dtype));
  };
  switch (st.kind) {
    case StepKind::JIT: {
      struct { void* p[48]; } args;
      std::memset(&args, 0, sizeof args);
      if (st.jit.ptrs.size() > 48) fail(PFC_ERR_UNSUPPORTED, "fused kernel with more than 48 operands");
      for (size_t k = 0; k < st.jit.ptrs.size(); ++k) args.p[k] = bufp(st.jit.ptrs[k].first, st.jit.ptrs[k].second);
      void* kargs[] = {&args};
      PFB_CUDA(cudaLaunchKernel((const void*)pe.kernels[i], dim3(st.jit.grid), dim3(st.jit.block), kargs,
                                st.jit.smem, s));
      break;
    }
    case StepKind::SPLIT: {
      const SplitArgs& a = st.split;
      PrepLaunch L;
      L.src = viewp(a.src);
      L.rank = (int)a.src.shape.size();
      if (L.rank > 6) fail(PFC_ERR_UNSUPPORTED, "matmul operand of rank > 6");
      for (int d = 0; d < L.rank; ++d) {
        L.shape[d] = a.src.shape[d];
        L.stride[d] = a.src.is_splat ? 0 : a.src.strides[d];
      }
      L.precision = a.precision;
      L.hi = bufp(a.out_hi, 0);
      L.lo = (float*)bufp(a.out_lo, 0);
      L.kpad = a.kpad;
      if (a.conv_cp > 0) {
        ConvWeightLaunch W;
        W.w = L.src;
        W.o = a.src.shape[0]; W.c = a.src.shape[1]; W.kh = a.src.shape[2]; W.kw = a.src.shape[3];
        W.so = L.stride[0]; W.sc = L.stride[1]; W.skh = L.stride[2]; W.skw = L.stride[3];
        W.cp = a.conv_cp; W.kpad = a.kpad; W.precision = a.precision; W.kwp = a.conv_kwp;
        W.hi = L.hi; W.lo = L.lo;
        launch_conv_weight(W, s);
      } else {
        launch_prepare(L, s);
      }
      break;
    }
    case StepKind::CONV_INPUT: {
      const ConvInputArgs& a = st.convin;
      ConvInputLaunch L;
      L.x = viewp(a.x);
      L.n = a.x.shape[0]; L.c = a.x.shape[1]; L.h = a.x.shape[2]; L.w = a.x.shape[3];
      L.sn = a.x.strides[0]; L.sc = a.x.strides[1]; L.sh = a.x.strides[2]; L.sw = a.x.strides[3];
      L.cp = a.cp; L.precision = a.precision;
      L.hp = a.hp; L.wp = a.wp; L.ph = a.ph; L.pw = a.pw;
      L.deint = a.deint;
      L.hi = bufp(a.out_hi, 0);
      L.lo = (float*)bufp(a.out_lo, 0);
      launch_conv_input(L, s);
      break;
    }
    case StepKind::IM2COL: {
      const Im2colArgs& a = st.im2col;
      Im2colLaunch L;
      L.x = viewp(a.x);
      L.n = a.x.shape[0]; L.c = a.x.shape[1]; L.h = a.x.shape[2]; L.w = a.x.shape[3];
      L.sn = a.x.strides[0]; L.sc = a.x.strides[1]; L.sh = a.x.strides[2]; L.sw = a.x.strides[3];
      L.kh = a.kh; L.kw = a.kw; L.stride_h = a.sh; L.stride_w = a.sw; L.pad_h = a.ph; L.pad_w = a.pw;
      L.dil_h = a.dh; L.dil_w = a.dw; L.oh = a.oh; L.ow = a.ow; L.kpad = a.kpad; L.precision = a.precision;
      L.hi = bufp(a.out_hi, 0);
      L.lo = (float*)bufp(a.out_lo, 0);
      launch_im2col(L, s);
      break;
    }
    case StepKind::ATTENTION: {
      const AttnArgs& a = st.attn;
      AttnLaunch L;
      L.precision = P.precision;
      L.batch = a.batch; L.M = a.M; L.L = a.L; L.d = a.d; L.kq = a.kq; L.kv = a.kv;
      L.q_hi = bufp(a.q_hi, 0);
      L.q_lo = (const float*)bufp(a.q_lo, 0);
      L.k_hi = bufp(a.k_hi, 0);
      L.k_lo = (const float*)bufp(a.k_lo, 0);
      L.v_hi = bufp(a.v_hi, 0);
      L.v_lo = (const float*)bufp(a.v_lo, 0);
      L.alpha = a.alpha;
      L.alpha_ptr = a.alpha_slot >= 0 ? (const float*)bufp(P.scalar_buf, (int64_t)a.alpha_slot * 4) : nullptr;
      const size_t r = a.c.shape.size();
      L.c = a.write_c ? (float*)viewp(a.c) : nullptr;
      L.heads = r == 4 ? a.c.shape[1] : 1;
      L.c_sb = a.c.strides[0];
      L.c_sh = r == 4 ? a.c.strides[1] : 0;
      L.c_sm = a.c.strides[r - 2];
      L.c_sn = a.c.strides[r - 1];
      if (a.op_hi >= 0) {
        // operand buffers share the element offsets of c
        const int64_t esz = P.precision == PFC_PRECISION_BF16 ? 2 : 4;
        L.o_hi = (float*)bufp(a.op_hi, a.c.offset * esz);
        L.o_lo = (float*)bufp(a.op_lo, a.c.offset * esz);
      }
      L.err = err_dev_;
      launch_attention(L, s);
      break;
    }
    case StepKind::GEMM: {
      const GemmArgs& a = st.gemm;
      GemmLaunch L;
      L.precision = a.precision;
      L.a_hi = bufp(a.a_hi, 0);
      L.a_lo = bufp(a.a_lo, 0);
      L.b_hi = bufp(a.b_hi, 0);
      L.b_lo = bufp(a.b_lo, 0);
      L.a_sb = a.a_sb; L.b_sb = a.b_sb; L.batch = a.batch; L.M = a.M; L.N = a.N; L.K = a.K; L.kpad = a.kpad;
      L.c = (float*)viewp(a.c);
      L.c_sb = a.c_sb; L.c_sm = a.c_sm; L.c_sn = a.c_sn;
      L.alpha = a.alpha;
      L.alpha_ptr = a.alpha_slot >= 0 ? (const float*)bufp(P.scalar_buf, (int64_t)a.alpha_slot * 4) : nullptr;
      if (a.has_bias) {
        if (a.bias.is_splat) L.bias_scalar = viewp(a.bias);
        else L.bias = viewp(a.bias);
      }
      L.scale = (const float*)bufp(a.scale_buf, 0);
      L.shift = (const float*)bufp(a.shift_buf, 0);
      L.act = a.act;
      if (a.has_residual) {
        L.residual = viewp(a.residual);
        L.r_sb = a.r_sb; L.r_sm = a.r_sm; L.r_sn = a.r_sn;
      }
      L.err = err_dev_;
      if (pe.tail) {
        L.tail_ws = (float*)pe.tail;
        L.tail_ws_bytes = (int64_t)tail_ws_bytes();
        L.tail_cnt = (unsigned*)((char*)pe.tail + tail_ws_bytes());
        L.tail_cnt_len = kTailCounters;
      }
      if (!a.write_c) L.c = nullptr;
      L.out_hi = bufp(a.op_hi, 0);
      L.out_lo = (float*)bufp(a.op_lo, 0);
      L.o_sm = a.op_sm;
      L.o_heads = a.op_heads;
      L.o_rows = a.op_rows;
      if (a.conv) {
        L.conv = true;
        L.x_hi = bufp(a.x_hi, 0);
        L.x_lo = bufp(a.x_lo, 0);
        L.H = a.H; L.W = a.W; L.Cp = a.Cp; L.KH = a.KH; L.KW = a.KW; L.sh = a.sh; L.sw = a.sw;
        L.ph = a.ph; L.pw = a.pw; L.dh = a.dh; L.dw = a.dw; L.OH = a.OH; L.OW = a.OW;
        L.batch_images = a.Nimg; L.Hp = a.Hp; L.Wp = a.Wp; L.KWp = a.KWp;
        L.deint = a.deint;
        if (a.pool) {
          L.pool = true;
          L.pool_pad = a.pool_pad;
          L.c = nullptr;
          L.pool_y = a.write_pool_y ? (float*)viewp(a.pool_y) : nullptr;
          L.pool_sn = a.pool_y.strides[0]; L.pool_sh = a.pool_y.strides[2]; L.pool_sw = a.pool_y.strides[3];
          L.PH = a.pool_y.shape[2]; L.PW = a.pool_y.shape[3];
        }
        if (a.gap_buf >= 0) {
          L.gap = (float*)bufp(a.gap_buf, 0);
          L.c = nullptr;
        }
      }
      launch_gemm(L, s);
      break;
    }
    case StepKind::POOL: {
      const PoolArgs& a = st.pool;
      PoolLaunch L;
      L.x = viewp(a.x);
      L.y = (float*)viewp(a.y);
      L.mode = a.mode;
      L.n = a.x.shape[0]; L.c = a.x.shape[1]; L.h = a.x.shape[2]; L.w = a.x.shape[3];
      L.sn = a.x.strides[0]; L.sc = a.x.strides[1]; L.sh = a.x.strides[2]; L.sw = a.x.strides[3];
      L.kh = a.kh; L.kw = a.kw; L.stride_h = a.sh; L.stride_w = a.sw; L.pad_h = a.ph; L.pad_w = a.pw;
      L.oh = a.y.shape[2]; L.ow = a.y.shape[3];
      L.osn = a.y.strides[0]; L.osc = a.y.strides[1]; L.osh = a.y.strides[2]; L.osw = a.y.strides[3];
      if (!a.write_y) L.y = nullptr;
      L.out_hi = bufp(a.op_hi, 0);
      L.out_lo = (float*)bufp(a.op_lo, 0);
      L.precision = P.precision;
      L.count = a.count;
      launch_pool(L, s);
      break;
    }
    case StepKind::BN_FOLD: {
      const BnFoldArgs& a = st.bnfold;
      BnFoldLaunch L;
      auto param = [&](const View& v, bool has, const float** p, int64_t* stride) {
        if (!has) return;
        *p = viewp(v);
        *stride = v.is_splat ? 0 : (v.strides.empty() ? 0 : v.strides.back());
        if (!v.is_splat) {
          for (size_t d = 0; d < v.shape.size(); ++d)
            if (v.shape[d] != 1) *stride = v.strides[d];
        }
      };
      param(a.gamma, a.has_gamma, &L.gamma, &L.gs);
      param(a.beta, a.has_beta, &L.beta, &L.bs);
      param(a.mean, true, &L.mean, &L.ms);
      param(a.var, true, &L.var, &L.vs);
      param(a.bias, a.has_bias, &L.bias, &L.cs);
      L.eps = a.eps;
      L.channels = a.channels;
      L.scale = (float*)bufp(a.out_scale, 0);
      L.shift = (float*)bufp(a.out_shift, 0);
      launch_bn_fold(L, s);
      break;
    }
    case StepKind::MEMSET:
      PFB_CUDA(cudaMemsetAsync(bufp(st.memset_buf, 0), 0, P.buffers[st.memset_buf].bytes, s));
      break;
    case StepKind::SMALL: {
      const SmallArgs& a = st.small;
      SmallMlpLaunch L;
      L.layers = a.layers;
      L.a = viewp(a.a);
      L.lda = a.lda;
      L.M = a.M;
      auto layer = [&](const SmallLayerArgs& l, const float** w, int64_t* ldw, const float** bias, int64_t* bstride,
                       float* alpha, const float** alpha_ptr, int* act) {
        *w = (const float*)bufp(l.w_buf, l.w_off * 4);
        *ldw = l.ldw;
        *bias = l.has_bias ? viewp(l.bias) : nullptr;
        *bstride = l.bstride;
        *alpha = l.alpha;
        *alpha_ptr = l.alpha_slot >= 0 ? (const float*)bufp(P.scalar_buf, (int64_t)l.alpha_slot * 4) : nullptr;
        *act = l.act;
      };
      layer(a.l1, &L.w1, &L.ldw1, &L.bias1, &L.bstride1, &L.alpha1, &L.alpha1_ptr, &L.act1);
      L.N1 = a.l1.N;
      L.K1 = a.l1.K;
      if (a.layers == 2) {
        layer(a.l2, &L.w2, &L.ldw2, &L.bias2, &L.bstride2, &L.alpha2, &L.alpha2_ptr, &L.act2);
        L.N2 = a.l2.N;
        L.h = (float*)bufp(a.h_buf, 0);
        L.ldh = a.l1.N;
        L.counter = (unsigned long long*)bufp(a.counter_buf, 0);
        L.cluster = a.cluster;
        L.err = err_dev_;
      }
      L.out = (float*)viewp(a.out);
      L.ldo = a.ldo;
      L.softmax = a.softmax;
      launch_small_mlp(L, s);
      break;
    }
  }
  if (cfg_.sync_after_launch) {
    PFB_CUDA(cudaStreamSynchronize(s));
    PFB_CUDA(cudaGetLastError());
  }
}

static int launches_of(const Step& s) { return s.kind == StepKind::MEMSET ? 0 : 1; }

int64_t CudaExecutor::run_steps(PlanEntry& pe, const std::vector<void*>& ptrs, cudaStream_t s) {
  const Plan& P = *pe.plan;
  int64_t launches = 0;
  // Operands derived from resident constants: prepared once, before (and
  // outside) the per-call sequence and its CUDA graph.
  for (size_t i = 0; i < P.steps.size(); ++i) {
    const Step& st = P.steps[i];
    if (!st.once) {
      launches += launches_of(st);
      continue;
    }
    Prepared& hi = prepared_.at(P.buffers[st.split.out_hi].prep_key);
    Prepared* lo = st.split.out_lo >= 0 ? &prepared_.at(P.buffers[st.split.out_lo].prep_key) : nullptr;
    if (hi.filled && (!lo || lo->filled)) continue;
    launch_step(pe, i, ptrs, s);
    launches += launches_of(st);
    hi.filled = true;
    if (lo) lo->filled = true;
  }
  profile_.clear();
  if (cfg_.enable_profiling) {
    std::vector<cudaEvent_t> ev(P.steps.size() + 1);
    for (auto& e : ev) PFB_CUDA(cudaEventCreate(&e));
    PFB_CUDA(cudaEventRecord(ev[0], s));
    for (size_t i = 0; i < P.steps.size(); ++i) {
      if (!P.steps[i].once) launch_step(pe, i, ptrs, s);
      PFB_CUDA(cudaEventRecord(ev[i + 1], s));
    }
    PFB_CUDA(cudaEventSynchronize(ev.back()));
    for (size_t i = 0; i < P.steps.size(); ++i) {
      if (P.steps[i].once) continue;
      float ms = 0;
      cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
      profile_.push_back({P.steps[i].label, (double)ms});
    }
    for (auto& e : ev) cudaEventDestroy(e);
    return launches;
  }
  bool graph_ok = cfg_.use_cuda_graph && !cfg_.sync_after_launch;
  if (graph_ok) {
    for (auto& gr : pe.graphs)
      if (gr.first == ptrs) {
        PFB_CUDA(cudaGraphLaunch(gr.second, s));
        ++pe.runs;
        return launches;
      }
  }
  if (graph_ok && pe.runs >= 1) {
    // capture once the plan has run eagerly (kernel attributes are set)
    constexpr size_t kGraphsPerPlan = 4;
    if (pe.graphs.size() >= kGraphsPerPlan) {
      cudaGraphExecDestroy(pe.graphs.front().second);
      pe.graphs.erase(pe.graphs.begin());
    }
    cudaGraphExec_t gexec = nullptr;
    cudaGraph_t graph;
    PFB_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    try {
      for (size_t i = 0; i < P.steps.size(); ++i)
        if (!P.steps[i].once) launch_step(pe, i, ptrs, s);
    } catch (...) {
      cudaStreamEndCapture(s, &graph);
      throw;
    }
    PFB_CUDA(cudaStreamEndCapture(s, &graph));
    cudaError_t e = cudaGraphInstantiate(&gexec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) {
      cudaGetLastError();
      for (size_t i = 0; i < P.steps.size(); ++i)
        if (!P.steps[i].once) launch_step(pe, i, ptrs, s);
    } else {
      pe.graphs.push_back({ptrs, gexec});
      PFB_CUDA(cudaGraphLaunch(gexec, s));
    }
    ++pe.runs;
    return launches;
  }
  for (size_t i = 0; i < P.steps.size(); ++i)
    if (!P.steps[i].once) launch_step(pe, i, ptrs, s);
  ++pe.runs;
  return launches;
}

void CudaExecutor::check_device_error(cudaStream_t s) {
  int h = 0;
  PFB_CUDA(cudaMemcpyAsync(&h, err_dev_, 4, cudaMemcpyDeviceToHost, s));
  PFB_CUDA(cudaStreamSynchronize(s));
  if (h != 0) {
    PFB_CUDA(cudaMemsetAsync(err_dev_, 0, 4, s));
    // a GEMM that stopped part-way may have left split-tail counters raised
    for (auto& kv : plans_)
      if (kv.second.tail)
        PFB_CUDA(cudaMemsetAsync((char*)kv.second.tail + tail_ws_bytes(), 0, kTailCounters * sizeof(unsigned), s));
    PFB_CUDA(cudaStreamSynchronize(s));
    fail(h, "a device-side bounded wait expired (tensor-core pipeline did not make progress)");
  }
}

void CudaExecutor::execute(Graph& g, const std::vector<uint64_t>& outs, void* const* host_out,
                           const size_t* out_bytes, pfc_execution_result* res) {
  std::lock_guard<std::mutex> lock(mu_);
  auto t0 = std::chrono::steady_clock::now();
  DeviceGuard dg(cfg_.device_id);
  h2d_ = 0;
  for (size_t i = 0; i < outs.size(); ++i) {
    const Node* n = g.find(outs[i]);
    if (!n) fail(PFC_ERR_INVALID_ARGUMENT, "output id " + std::to_string(outs[i]) + " is not in the graph");
    if (!host_out[i]) fail(PFC_ERR_INVALID_ARGUMENT, "null output buffer");
    if (out_bytes[i] != n->size_bytes())
      fail(PFC_ERR_INVALID_ARGUMENT, "output buffer for node " + std::to_string(outs[i]) + " has " +
                                         std::to_string(out_bytes[i]) + " bytes, expected " +
                                         std::to_string(n->size_bytes()));
  }
  double compile_ms = 0;
  PlanEntry& pe = prepare(g, outs, {}, &compile_ms);
  const Plan& P = *pe.plan;
  cudaStream_t s = stream_;
  cudaEvent_t e0, e1, e2, e3;
  PFB_CUDA(cudaEventCreate(&e0));
  PFB_CUDA(cudaEventCreate(&e1));
  PFB_CUDA(cudaEventCreate(&e2));
  PFB_CUDA(cudaEventCreate(&e3));
  PFB_CUDA(cudaEventRecord(e0, s));
  std::vector<std::pair<void*, const Node*>> uploads;
  std::vector<void*> ptrs = resolve(pe, g, {}, s, &uploads);
  for (auto& [dst, n] : uploads) {
    PFB_CUDA(cudaMemcpyAsync(dst, n->data, n->data_bytes, cudaMemcpyHostToDevice, s));
    h2d_ += n->data_bytes;
  }
  {
    // splat values live in a small device table; upload only when they change
    std::vector<float> table(P.scalars.size());
    for (size_t i = 0; i < P.scalars.size(); ++i) table[i] = P.scalars[i].value;
    if (!table.empty() && (table != pe.table || pe.table_ptr != ptrs[P.scalar_buf])) {
      PFB_CUDA(cudaMemcpyAsync(ptrs[P.scalar_buf], table.data(), table.size() * 4, cudaMemcpyHostToDevice, s));
      h2d_ += table.size() * 4;
      pe.table = table;
      pe.table_ptr = ptrs[P.scalar_buf];
    }
  }
  PFB_CUDA(cudaEventRecord(e1, s));
  int64_t launches = run_steps(pe, ptrs, s);
  PFB_CUDA(cudaEventRecord(e2, s));
  for (size_t i = 0; i < outs.size(); ++i) {
    const View& v = P.output_views[i];
    const void* src = (const char*)ptrs[v.buf] + v.offset * (int64_t)dtype_size(v.dtype);
    if (out_bytes[i]) PFB_CUDA(cudaMemcpyAsync(host_out[i], src, out_bytes[i], cudaMemcpyDeviceToHost, s));
  }
  PFB_CUDA(cudaEventRecord(e3, s));
  cudaError_t se = cudaStreamSynchronize(s);
  if (se != cudaSuccess) fail(PFC_ERR_CUDA, std::string("execution failed: ") + cudaGetErrorString(se));
  check_device_error(s);
  float up = 0, comp = 0, down = 0;
  cudaEventElapsedTime(&up, e0, e1);
  cudaEventElapsedTime(&comp, e1, e2);
  cudaEventElapsedTime(&down, e2, e3);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaEventDestroy(e2);
  cudaEventDestroy(e3);
  res->success = 1;
  res->compile_time_ms = compile_ms;
  res->transfer_time_ms = up + down;
  res->compute_time_ms = comp;
  res->total_time_ms = ms_since(t0);
  res->kernel_launches = launches;
  res->h2d_bytes = h2d_;
  res->d2h_bytes = [&] {
    uint64_t b = 0;
    for (size_t i = 0; i < outs.size(); ++i) b += out_bytes[i];
    return b;
  }();
}

void CudaExecutor::execute_device(Graph& g, const std::vector<uint64_t>& in_ids, const void* const* in_dev,
                                  const std::vector<uint64_t>& outs, void* const* out_dev, cudaStream_t stream,
                                  pfc_execution_result* res) {
  std::lock_guard<std::mutex> lock(mu_);
  auto t0 = std::chrono::steady_clock::now();
  DeviceGuard dg(cfg_.device_id);
  h2d_ = 0;
  std::unordered_set<uint64_t> bindings;
  std::unordered_map<uint64_t, const void*> bind;
  for (size_t i = 0; i < in_ids.size(); ++i) {
    const Node* n = g.find(in_ids[i]);
    if (!n) fail(PFC_ERR_INVALID_ARGUMENT, "input id " + std::to_string(in_ids[i]) + " is not in the graph");
    if (n->type == NodeType::OPERATION) fail(PFC_ERR_INVALID_ARGUMENT, "only leaf nodes can be bound to device data");
    if (((uintptr_t)in_dev[i] & 15) != 0) fail(PFC_ERR_INVALID_ARGUMENT, "device input pointers must be 16-byte aligned");
    bindings.insert(in_ids[i]);
    bind[in_ids[i]] = in_dev[i];
  }
  for (size_t i = 0; i < outs.size(); ++i)
    if (!g.find(outs[i])) fail(PFC_ERR_INVALID_ARGUMENT, "output id " + std::to_string(outs[i]) + " is not in the graph");
  double compile_ms = 0;
  PlanEntry& pe = prepare(g, outs, bindings, &compile_ms);
  const Plan& P = *pe.plan;
  cudaStream_t s = stream ? stream : stream_;
  std::vector<std::pair<void*, const Node*>> uploads;
  std::vector<void*> ptrs = resolve(pe, g, bind, s, &uploads);
  // Outputs whose buffer is exclusively theirs are written in place.
  std::vector<bool> direct(outs.size(), false);
  std::unordered_map<int, int> owner;
  for (size_t i = 0; i < outs.size(); ++i) owner[P.output_views[i].buf]++;
  for (size_t i = 0; i < outs.size(); ++i) {
    const View& v = P.output_views[i];
    const Buffer& b = P.buffers[v.buf];
    if (b.kind == BufKind::ARENA && v.offset == 0 && owner[v.buf] == 1 && ((uintptr_t)out_dev[i] & 255) == 0) {
      ptrs[v.buf] = out_dev[i];
      direct[i] = true;
    }
  }
  for (auto& [dst, n] : uploads) {
    PFB_CUDA(cudaMemcpyAsync(dst, n->data, n->data_bytes, cudaMemcpyHostToDevice, s));
    h2d_ += n->data_bytes;
  }
  {
    // splat values live in a small device table; upload only when they change
    std::vector<float> table(P.scalars.size());
    for (size_t i = 0; i < P.scalars.size(); ++i) table[i] = P.scalars[i].value;
    if (!table.empty() && (table != pe.table || pe.table_ptr != ptrs[P.scalar_buf])) {
      PFB_CUDA(cudaMemcpyAsync(ptrs[P.scalar_buf], table.data(), table.size() * 4, cudaMemcpyHostToDevice, s));
      h2d_ += table.size() * 4;
      pe.table = table;
      pe.table_ptr = ptrs[P.scalar_buf];
    }
  }
  int64_t launches = run_steps(pe, ptrs, s);
  for (size_t i = 0; i < outs.size(); ++i) {
    if (direct[i]) continue;
    const View& v = P.output_views[i];
    const void* src = (const char*)ptrs[v.buf] + v.offset * (int64_t)dtype_size(v.dtype);
    PFB_CUDA(cudaMemcpyAsync(out_dev[i], src, g.at(outs[i]).size_bytes(), cudaMemcpyDeviceToDevice, s));
  }
  res->success = 1;
  res->compile_time_ms = compile_ms;
  res->total_time_ms = ms_since(t0);
  res->kernel_launches = launches;
  res->h2d_bytes = h2d_;
  res->d2h_bytes = 0;
}

void CudaExecutor::execute_streamed(Graph& g, const std::vector<uint64_t>& in_ids, const void* const* in_host,
                                    const std::vector<uint64_t>& outs, void* const* out_host, int n_chunks,
                                    pfc_execution_result* res) {
  std::lock_guard<std::mutex> lock(mu_);
  auto t0 = std::chrono::steady_clock::now();
  DeviceGuard dg(cfg_.device_id);
  h2d_ = 0;
  if (n_chunks < 1) fail(PFC_ERR_INVALID_ARGUMENT, "n_chunks must be at least 1");
  std::unordered_set<uint64_t> bindings;
  std::vector<size_t> in_bytes, out_bytes;
  for (size_t i = 0; i < in_ids.size(); ++i) {
    const Node* n = g.find(in_ids[i]);
    if (!n) fail(PFC_ERR_INVALID_ARGUMENT, "input id " + std::to_string(in_ids[i]) + " is not in the graph");
    if (n->type == NodeType::OPERATION) fail(PFC_ERR_INVALID_ARGUMENT, "only leaf nodes can be streamed inputs");
    if (!in_host[i]) fail(PFC_ERR_INVALID_ARGUMENT, "null input buffer");
    bindings.insert(in_ids[i]);
    in_bytes.push_back(n->size_bytes());
  }
  for (size_t i = 0; i < outs.size(); ++i) {
    const Node* n = g.find(outs[i]);
    if (!n) fail(PFC_ERR_INVALID_ARGUMENT, "output id " + std::to_string(outs[i]) + " is not in the graph");
    if (!out_host[i]) fail(PFC_ERR_INVALID_ARGUMENT, "null output buffer");
    out_bytes.push_back(n->size_bytes());
  }
  double compile_ms = 0;
  PlanEntry& pe = prepare(g, outs, bindings, &compile_ms);
  const Plan& P = *pe.plan;
  if (!copy_in_) PFB_CUDA(cudaStreamCreateWithFlags(&copy_in_, cudaStreamNonBlocking));
  if (!copy_out_) PFB_CUDA(cudaStreamCreateWithFlags(&copy_out_, cudaStreamNonBlocking));
  // two device slots per input and output, kept with the plan between calls
  const cudaStream_t s = stream_;
  std::vector<size_t> want(in_bytes);
  want.insert(want.end(), out_bytes.begin(), out_bytes.end());
  if (pe.slot_bytes != want) {
    PFB_CUDA(cudaStreamSynchronize(s));
    for (int k = 0; k < 2; ++k) {
      for (void* p : pe.slots[k]) PFB_CUDA(pool_->deallocate(p, s));
      pe.slots[k].clear();
      for (size_t b : want) pe.slots[k].push_back(pool_->allocate(std::max<size_t>(b, 256), s));
    }
    pe.slot_bytes = want;
  }
  std::vector<void*> in_slot[2], out_slot[2];
  for (int k = 0; k < 2; ++k) {
    in_slot[k].assign(pe.slots[k].begin(), pe.slots[k].begin() + in_bytes.size());
    out_slot[k].assign(pe.slots[k].begin() + in_bytes.size(), pe.slots[k].end());
  }
  cudaEvent_t ready, ev_in[2], ev_comp[2], ev_out[2], e_start, e_end;
  PFB_CUDA(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
  for (int k = 0; k < 2; ++k) {
    PFB_CUDA(cudaEventCreateWithFlags(&ev_in[k], cudaEventDisableTiming));
    PFB_CUDA(cudaEventCreateWithFlags(&ev_comp[k], cudaEventDisableTiming));
    PFB_CUDA(cudaEventCreateWithFlags(&ev_out[k], cudaEventDisableTiming));
  }
  PFB_CUDA(cudaEventCreate(&e_start));
  PFB_CUDA(cudaEventCreate(&e_end));
  PFB_CUDA(cudaEventRecord(ready, s));  // slots exist
  PFB_CUDA(cudaStreamWaitEvent(copy_in_, ready));
  PFB_CUDA(cudaStreamWaitEvent(copy_out_, ready));
  PFB_CUDA(cudaEventRecord(e_start, copy_in_));
  int64_t launches = 0;
  std::unordered_map<int, int> owner;
  for (size_t i = 0; i < outs.size(); ++i) owner[P.output_views[i].buf]++;
  for (int c = 0; c < n_chunks; ++c) {
    const int k = c & 1;
    // inputs of chunk c into slot k once chunk c-2 has finished reading it
    if (c >= 2) PFB_CUDA(cudaStreamWaitEvent(copy_in_, ev_comp[k]));
    for (size_t i = 0; i < in_ids.size(); ++i)
    {
      PFB_CUDA(cudaMemcpyAsync(in_slot[k][i], (const char*)in_host[i] + (size_t)c * in_bytes[i], in_bytes[i],
                               cudaMemcpyHostToDevice, copy_in_));
      h2d_ += in_bytes[i];
    }
    PFB_CUDA(cudaEventRecord(ev_in[k], copy_in_));
    // compute chunk c once its inputs landed and chunk c-2's outputs left slot k
    PFB_CUDA(cudaStreamWaitEvent(s, ev_in[k]));
    if (c >= 2) PFB_CUDA(cudaStreamWaitEvent(s, ev_out[k]));
    std::unordered_map<uint64_t, const void*> bind;
    for (size_t i = 0; i < in_ids.size(); ++i) bind[in_ids[i]] = in_slot[k][i];
    std::vector<std::pair<void*, const Node*>> uploads;
    std::vector<void*> ptrs = resolve(pe, g, bind, s, &uploads);
    std::vector<bool> direct(outs.size(), false);
    for (size_t i = 0; i < outs.size(); ++i) {
      const View& v = P.output_views[i];
      const Buffer& b = P.buffers[v.buf];
      if (b.kind == BufKind::ARENA && v.offset == 0 && owner[v.buf] == 1) {
        ptrs[v.buf] = out_slot[k][i];
        direct[i] = true;
      }
    }
    for (auto& [dst, n] : uploads) {
    PFB_CUDA(cudaMemcpyAsync(dst, n->data, n->data_bytes, cudaMemcpyHostToDevice, s));
    h2d_ += n->data_bytes;
  }
    {
      std::vector<float> table(P.scalars.size());
      for (size_t i = 0; i < P.scalars.size(); ++i) table[i] = P.scalars[i].value;
      if (!table.empty() && (table != pe.table || pe.table_ptr != ptrs[P.scalar_buf])) {
        PFB_CUDA(cudaMemcpyAsync(ptrs[P.scalar_buf], table.data(), table.size() * 4, cudaMemcpyHostToDevice, s));
      h2d_ += table.size() * 4;
        pe.table = table;
        pe.table_ptr = ptrs[P.scalar_buf];
      }
    }
    launches += run_steps(pe, ptrs, s);
    for (size_t i = 0; i < outs.size(); ++i) {
      if (direct[i]) continue;
      const View& v = P.output_views[i];
      const void* src = (const char*)ptrs[v.buf] + v.offset * (int64_t)dtype_size(v.dtype);
      PFB_CUDA(cudaMemcpyAsync(out_slot[k][i], src, out_bytes[i], cudaMemcpyDeviceToDevice, s));
    }
    PFB_CUDA(cudaEventRecord(ev_comp[k], s));
    // outputs of chunk c back to the host
    PFB_CUDA(cudaStreamWaitEvent(copy_out_, ev_comp[k]));
    for (size_t i = 0; i < outs.size(); ++i)
      PFB_CUDA(cudaMemcpyAsync((char*)out_host[i] + (size_t)c * out_bytes[i], out_slot[k][i], out_bytes[i],
                               cudaMemcpyDeviceToHost, copy_out_));
    PFB_CUDA(cudaEventRecord(ev_out[k], copy_out_));
  }
  PFB_CUDA(cudaEventRecord(e_end, copy_out_));
  cudaError_t se = cudaStreamSynchronize(copy_out_);
  if (se == cudaSuccess) se = cudaStreamSynchronize(s);
  float total = 0;
  if (se == cudaSuccess) cudaEventElapsedTime(&total, e_start, e_end);
  // the next call's first copies must not overtake this call's last reads
  PFB_CUDA(cudaEventRecord(ready, copy_in_));
  PFB_CUDA(cudaStreamWaitEvent(s, ready));
  cudaEventDestroy(ready);
  for (int k = 0; k < 2; ++k) {
    cudaEventDestroy(ev_in[k]);
    cudaEventDestroy(ev_comp[k]);
    cudaEventDestroy(ev_out[k]);
  }
  cudaEventDestroy(e_start);
  cudaEventDestroy(e_end);
  if (se != cudaSuccess) fail(PFC_ERR_CUDA, std::string("execution failed: ") + cudaGetErrorString(se));
  check_device_error(s);
  res->success = 1;
  res->compile_time_ms = compile_ms;
  res->transfer_time_ms = total;  // copies overlap compute: the span of the whole pipeline
  res->compute_time_ms = total;
  res->total_time_ms = ms_since(t0);
  res->kernel_launches = launches;
  res->h2d_bytes = h2d_;
  res->d2h_bytes = [&] {
    uint64_t b = 0;
    for (size_t i = 0; i < outs.size(); ++i) b += out_bytes[i];
    return b * (uint64_t)n_chunks;
  }();
}

std::string CudaExecutor::describe(Graph& g, const std::vector<uint64_t>& outs) {
  std::lock_guard<std::mutex> lock(mu_);
  DeviceGuard dg(cfg_.device_id);
  PlanEntry& pe = prepare(g, outs, {}, nullptr);
  return pe.plan->description;
}

}  // namespace pfb
