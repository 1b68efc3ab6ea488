// extern "C" surface of include/pyflame_cuda.h.  Every entry point catches
// all exceptions and turns them into a PFC_ERR_* code plus a thread-local
// message (PyFlame's executors report failures the same way:
// executor.cpp:212-275, rocm_executor.cpp:75-154).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>

#include "../../include/pyflame_cuda.h"
#include "common.hpp"
#include "executor.hpp"
#include "graph.hpp"
#include "jit.hpp"
#include "kernels/kernels.hpp"

struct pfc_graph {
  pfb::Graph g;
};
struct pfc_executor {
  std::unique_ptr<pfb::CudaExecutor> ex;
};

namespace pfb {
static thread_local std::string t_last_error;
void set_last_error(const std::string& msg) { t_last_error = msg; }
}  // namespace pfb

namespace {

template <class F>
int guarded(F&& f) {
  try {
    f();
    return PFC_OK;
  } catch (const pfb::Error& e) {
    pfb::set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    pfb::set_last_error("host allocation failed");
    return PFC_ERR_OUT_OF_MEMORY;
  } catch (const std::exception& e) {
    pfb::set_last_error(e.what());
    return PFC_ERR_INTERNAL;
  } catch (...) {
    pfb::set_last_error("unknown error");
    return PFC_ERR_INTERNAL;
  }
}

void fill_error(pfc_execution_result* r, int code) {
  if (!r) return;
  r->success = 0;
  std::snprintf(r->error_message, sizeof r->error_message, "%s", pfb::t_last_error.c_str());
  (void)code;
}

cudaStream_t as_stream(void* s) { return (cudaStream_t)s; }

}  // namespace

extern "C" {

const char* pfc_last_error(void) { return pfb::t_last_error.c_str(); }
int pfc_abi_version(void) { return PFC_ABI_VERSION; }

// ---- device functions --------------------------------------------------------
int pfc_cuda_is_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  for (int d = 0; d < n; ++d) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) == cudaSuccess && major >= 10) return 1;
  }
  return 0;
}

int pfc_cuda_get_device_count(int* count) {
  return guarded([&] {
    PFB_CHECK_ARG(count, "null count");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    *count = n;
  });
}

int pfc_cuda_get_device_info(int device_id, pfc_device_info* info) {
  return guarded([&] {
    PFB_CHECK_ARG(info, "null info");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device_id < 0 || device_id >= n) {
      cudaGetLastError();
      pfb::fail(PFC_ERR_NO_DEVICE, "Invalid device ID: " + std::to_string(device_id));
    }
    cudaDeviceProp p;
    PFB_CUDA(cudaGetDeviceProperties(&p, device_id));
    std::memset(info, 0, sizeof *info);
    info->device_id = device_id;
    std::snprintf(info->name, sizeof info->name, "%s", p.name);
    std::snprintf(info->architecture, sizeof info->architecture, "sm_%d%d", p.major, p.minor);
    info->total_memory = p.totalGlobalMem;
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur == device_id) {
      size_t fr = 0, tot = 0;
      if (cudaMemGetInfo(&fr, &tot) == cudaSuccess) info->free_memory = fr;
      else cudaGetLastError();
    }
    info->compute_units = p.multiProcessorCount;
    info->max_threads_per_block = p.maxThreadsPerBlock;
    info->warp_size = p.warpSize;
  });
}

int pfc_cuda_set_device(int device_id) {
  return guarded([&] {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device_id < 0 || device_id >= n) {
      cudaGetLastError();
      pfb::fail(PFC_ERR_NO_DEVICE, "Invalid device ID: " + std::to_string(device_id));
    }
    PFB_CUDA(cudaSetDevice(device_id));
  });
}

int pfc_cuda_get_device(int* device_id) {
  return guarded([&] {
    PFB_CHECK_ARG(device_id, "null device_id");
    PFB_CUDA(cudaGetDevice(device_id));
  });
}

int pfc_cuda_synchronize(void) {
  return guarded([&] { PFB_CUDA(cudaDeviceSynchronize()); });
}

// ---- graph description -------------------------------------------------------
int pfc_graph_create(pfc_graph** out) {
  return guarded([&] {
    PFB_CHECK_ARG(out, "null out");
    *out = new pfc_graph();
  });
}

int pfc_graph_destroy(pfc_graph* g) {
  delete g;
  return PFC_OK;
}

int pfc_graph_add_node(pfc_graph* g, uint64_t id, int node_type, int op_type, int dtype, int ndim,
                       const int64_t* shape, int n_inputs, const uint64_t* input_ids) {
  return guarded([&] {
    PFB_CHECK_ARG(g, "null graph");
    PFB_CHECK_ARG(node_type >= 0 && node_type <= 3, "bad node type");
    PFB_CHECK_ARG(dtype >= 0 && dtype <= 8, "bad dtype");
    PFB_CHECK_ARG(ndim >= 0 && ndim <= 64 && (ndim == 0 || shape), "bad shape");
    PFB_CHECK_ARG(n_inputs >= 0 && (n_inputs == 0 || input_ids), "bad inputs");
    PFB_CHECK_ARG(!g->g.index.count(id), "duplicate node id " + std::to_string(id));
    pfb::Node n;
    n.id = id;
    n.type = (pfb::NodeType)node_type;
    n.op = (pfb::Op)op_type;
    n.dtype = (pfb::DType)dtype;
    n.shape.assign(shape, shape + ndim);
    for (int64_t d : n.shape) PFB_CHECK_ARG(d >= 0, "negative dimension");
    n.inputs.assign(input_ids, input_ids + n_inputs);
    g->g.index[id] = g->g.nodes.size();
    g->g.nodes.push_back(std::move(n));
    g->g.version++;
  });
}

int pfc_graph_set_attr(pfc_graph* g, uint64_t id, const char* key, int attr_type, const void* value,
                       int64_t count) {
  return guarded([&] {
    PFB_CHECK_ARG(g && key && value, "null argument");
    pfb::Node* n = g->g.find(id);
    PFB_CHECK_ARG(n, "no node " + std::to_string(id));
    pfb::Attr a;
    a.type = attr_type;
    switch (attr_type) {
      case PFC_ATTR_INT32: a.i.push_back(*(const int32_t*)value); break;
      case PFC_ATTR_INT64: a.i.push_back(*(const int64_t*)value); break;
      case PFC_ATTR_BOOL: a.i.push_back(*(const uint8_t*)value ? 1 : 0); break;
      case PFC_ATTR_FLOAT32: a.f.push_back(*(const float*)value); break;
      case PFC_ATTR_FLOAT64: a.f.push_back(*(const double*)value); break;
      case PFC_ATTR_INT64_VEC:
        PFB_CHECK_ARG(count >= 0, "negative count");
        for (int64_t i = 0; i < count; ++i) a.i.push_back(((const int64_t*)value)[i]);
        break;
      case PFC_ATTR_INT32_VEC:
        PFB_CHECK_ARG(count >= 0, "negative count");
        for (int64_t i = 0; i < count; ++i) a.i.push_back(((const int32_t*)value)[i]);
        break;
      case PFC_ATTR_FLOAT32_VEC:
        PFB_CHECK_ARG(count >= 0, "negative count");
        for (int64_t i = 0; i < count; ++i) a.f.push_back(((const float*)value)[i]);
        break;
      default: pfb::fail(PFC_ERR_INVALID_ARGUMENT, "bad attribute type");
    }
    n->attrs[key] = std::move(a);
    g->g.version++;
  });
}

int pfc_graph_set_constant(pfc_graph* g, uint64_t id, const void* data, size_t bytes, uint32_t flags,
                           uint64_t cache_key) {
  return guarded([&] {
    PFB_CHECK_ARG(g, "null graph");
    pfb::Node* n = g->g.find(id);
    PFB_CHECK_ARG(n, "no node " + std::to_string(id));
    PFB_CHECK_ARG(bytes == 0 || data, "null data");
    // Graph::create_constant copies spec.size_bytes() (graph.hpp:40-45)
    PFB_CHECK_ARG(bytes == n->size_bytes(), "constant payload of node " + std::to_string(id) + " has " +
                                                std::to_string(bytes) + " bytes, expected " +
                                                std::to_string(n->size_bytes()));
    if (flags & PFC_CONST_COPY) {
      n->owned.assign((const uint8_t*)data, (const uint8_t*)data + bytes);
      n->data = n->owned.data();
    } else {
      n->owned.clear();
      n->data = data;
    }
    n->data_bytes = bytes;
    n->data_flags = flags;
    n->data_key = cache_key ? cache_key : (uint64_t)(uintptr_t)data;
    g->g.version++;
  });
}

int pfc_graph_mark_output(pfc_graph* g, uint64_t id) {
  return guarded([&] {
    PFB_CHECK_ARG(g && g->g.find(id), "no node " + std::to_string(id));
    for (uint64_t o : g->g.outputs)
      if (o == id) return;
    g->g.outputs.push_back(id);
  });
}

int pfc_graph_num_nodes(const pfc_graph* g, int64_t* n) {
  return guarded([&] {
    PFB_CHECK_ARG(g && n, "null argument");
    *n = (int64_t)g->g.nodes.size();
  });
}

// ---- executor ------------------------------------------------------------------
void pfc_executor_config_default(pfc_executor_config* cfg) {
  if (!cfg) return;
  std::memset(cfg, 0, sizeof *cfg);
  cfg->device_id = 0;
  cfg->workspace_size_mb = 256;
  cfg->precision = PFC_PRECISION_TF32X3;
  cfg->use_cuda_graph = 1;
}

int pfc_executor_create(const pfc_executor_config* cfg, pfc_executor** out) {
  return guarded([&] {
    PFB_CHECK_ARG(out, "null out");
    pfc_executor_config c;
    if (cfg) c = *cfg;
    else pfc_executor_config_default(&c);
    PFB_CHECK_ARG(c.precision == PFC_PRECISION_TF32X3 || c.precision == PFC_PRECISION_BF16, "bad precision");
    auto e = std::make_unique<pfc_executor>();
    e->ex = std::make_unique<pfb::CudaExecutor>(c);
    *out = e.release();
  });
}

int pfc_executor_destroy(pfc_executor* ex) {
  return guarded([&] { delete ex; });
}

int pfc_executor_execute(pfc_executor* ex, pfc_graph* g, const uint64_t* output_ids, int n_outputs,
                         void* const* out_host, const size_t* out_bytes, pfc_execution_result* result) {
  if (result) std::memset(result, 0, sizeof *result);
  int rc = guarded([&] {
    PFB_CHECK_ARG(ex && g && result, "null argument");
    PFB_CHECK_ARG(n_outputs >= 0 && (n_outputs == 0 || (output_ids && out_host && out_bytes)), "bad outputs");
    std::vector<uint64_t> outs(output_ids, output_ids + n_outputs);
    ex->ex->execute(g->g, outs, out_host, out_bytes, result);
  });
  if (rc != PFC_OK) fill_error(result, rc);
  return rc;
}

int pfc_executor_execute_device(pfc_executor* ex, pfc_graph* g, const uint64_t* input_ids, int n_inputs,
                                const void* const* in_dev, const uint64_t* output_ids, int n_outputs,
                                void* const* out_dev, void* stream, pfc_execution_result* result) {
  if (result) std::memset(result, 0, sizeof *result);
  int rc = guarded([&] {
    PFB_CHECK_ARG(ex && g && result, "null argument");
    PFB_CHECK_ARG(n_inputs >= 0 && (n_inputs == 0 || (input_ids && in_dev)), "bad inputs");
    PFB_CHECK_ARG(n_outputs >= 0 && (n_outputs == 0 || (output_ids && out_dev)), "bad outputs");
    std::vector<uint64_t> ins(input_ids, input_ids + n_inputs), outs(output_ids, output_ids + n_outputs);
    ex->ex->execute_device(g->g, ins, in_dev, outs, out_dev, as_stream(stream), result);
  });
  if (rc != PFC_OK) fill_error(result, rc);
  return rc;
}

int pfc_executor_execute_streamed(pfc_executor* ex, pfc_graph* g, const uint64_t* input_ids, int n_inputs,
                                  const void* const* in_host, const uint64_t* output_ids, int n_outputs,
                                  void* const* out_host, int n_chunks, pfc_execution_result* result) {
  if (result) std::memset(result, 0, sizeof *result);
  int rc = guarded([&] {
    PFB_CHECK_ARG(ex && g && result, "null argument");
    PFB_CHECK_ARG(n_inputs >= 0 && (n_inputs == 0 || (input_ids && in_host)), "bad inputs");
    PFB_CHECK_ARG(n_outputs > 0 && output_ids && out_host, "bad outputs");
    std::vector<uint64_t> ins(input_ids, input_ids + n_inputs), outs(output_ids, output_ids + n_outputs);
    ex->ex->execute_streamed(g->g, ins, in_host, outs, out_host, n_chunks, result);
  });
  if (rc != PFC_OK) fill_error(result, rc);
  return rc;
}

int pfc_executor_get_device_info(pfc_executor* ex, pfc_device_info* info) {
  return guarded([&] {
    PFB_CHECK_ARG(ex && info, "null argument");
    *info = ex->ex->device_info();
  });
}

int pfc_executor_get_memory_stats(pfc_executor* ex, pfc_memory_stats* stats) {
  return guarded([&] {
    PFB_CHECK_ARG(ex && stats, "null argument");
    *stats = ex->ex->memory_stats();
  });
}

int pfc_executor_release_constants(pfc_executor* ex) {
  return guarded([&] {
    PFB_CHECK_ARG(ex, "null executor");
    PFB_CUDA(ex->ex->release_constants());
  });
}

int pfc_executor_set_resident(pfc_executor* ex, uint64_t cache_key, const void* dev_ptr, size_t bytes) {
  return guarded([&] {
    PFB_CHECK_ARG(ex, "null executor");
    ex->ex->set_resident(cache_key, dev_ptr, bytes);
  });
}

int pfc_executor_describe_plan(pfc_executor* ex, pfc_graph* g, const uint64_t* output_ids, int n_outputs,
                               char* buf, size_t buf_len) {
  return guarded([&] {
    PFB_CHECK_ARG(ex && g && buf && buf_len, "null argument");
    std::vector<uint64_t> outs(output_ids, output_ids + n_outputs);
    std::string d = ex->ex->describe(g->g, outs);
    std::snprintf(buf, buf_len, "%s", d.c_str());
  });
}

int pfc_compile_check(pfc_graph* g, const uint64_t* output_ids, int n_outputs, int precision, char* buf,
                      size_t buf_len) {
  return guarded([&] {
    PFB_CHECK_ARG(g && buf && buf_len && (n_outputs == 0 || output_ids), "null argument");
    std::vector<uint64_t> outs(output_ids, output_ids + n_outputs);
    pfb::validate_graph(g->g);
    auto order = pfb::topo_order(g->g, outs);
    pfb::CompileInput ci;
    ci.g = &g->g;
    ci.outputs = outs;
    ci.splats = pfb::detect_splats(g->g, order, {});
    ci.precision = precision;
    ci.num_sms = 148;
    pfb::SourceMap sources;
    auto plan = pfb::compile_plan(ci, &sources);
    std::string desc = plan->description;
    const char* dump = std::getenv("PFB_DUMP_DIR");
    for (auto& [key, src] : sources) {
      if (dump) {
        std::string path = std::string(dump) + "/" + key + ".cu";
        if (FILE* f = std::fopen(path.c_str(), "w")) {
          std::fwrite(src.first.data(), 1, src.first.size(), f);
          std::fclose(f);
        }
      }
      std::string log;
      size_t n = pfb::JitCache::compile_only(src.first, &log);
      desc += "  kernel " + key + ": cubin " + std::to_string(n) + " bytes\n";
    }
    std::snprintf(buf, buf_len, "%s", desc.c_str());
  });
}

int pfc_executor_last_profile(pfc_executor* ex, char (*names)[64], double* ms, int cap, int* count) {
  return guarded([&] {
    PFB_CHECK_ARG(ex && count, "null argument");
    const auto& p = ex->ex->last_profile();
    int n = 0;
    for (const auto& [name, t] : p) {
      if (n >= cap) break;
      if (names) std::snprintf(names[n], 64, "%s", name.c_str());
      if (ms) ms[n] = t;
      ++n;
    }
    *count = (int)p.size();
  });
}

// ---- kernel entry points ---------------------------------------------------------
int pfk_check_bounded_wait(int* err, int64_t limit_us, void* stream) {
  return guarded([&] { pfb::launch_wait_check(err, limit_us, (cudaStream_t)stream); });
}

int pfk_split_tf32(const float* src, int64_t batch, int64_t rows, int64_t cols, int64_t sb, int64_t sr, int64_t sk,
                   float* hi, float* lo, int64_t kpad, void* stream) {
  return guarded([&] {
    PFB_CHECK_ARG(src && hi && lo, "null pointer");
    PFB_CHECK_ARG(kpad >= cols && kpad % 4 == 0, "kpad must be >= cols and a multiple of 4");
    pfb::PrepLaunch L;
    L.src = src;
    L.rank = 3;
    L.shape[0] = batch; L.shape[1] = rows; L.shape[2] = cols;
    L.stride[0] = sb; L.stride[1] = sr; L.stride[2] = sk;
    L.precision = PFC_PRECISION_TF32X3;
    L.hi = hi;
    L.lo = lo;
    L.kpad = kpad;
    pfb::launch_prepare(L, as_stream(stream));
  });
}

int pfk_convert_bf16(const float* src, int64_t batch, int64_t rows, int64_t cols, int64_t sb, int64_t sr,
                     int64_t sk, uint16_t* out, int64_t kpad, void* stream) {
  return guarded([&] {
    PFB_CHECK_ARG(src && out, "null pointer");
    PFB_CHECK_ARG(kpad >= cols && kpad % 4 == 0, "kpad must be >= cols and a multiple of 4");
    pfb::PrepLaunch L;
    L.src = src;
    L.rank = 3;
    L.shape[0] = batch; L.shape[1] = rows; L.shape[2] = cols;
    L.stride[0] = sb; L.stride[1] = sr; L.stride[2] = sk;
    L.precision = PFC_PRECISION_BF16;
    L.hi = out;
    L.kpad = kpad;
    pfb::launch_prepare(L, as_stream(stream));
  });
}

int pfk_gemm(int precision, const void* a_hi, const void* a_lo, int64_t a_sb, const void* b_hi, const void* b_lo,
             int64_t b_sb, int64_t batch, int64_t M, int64_t N, int64_t K, int64_t kpad, float* c, int64_t c_sb,
             int64_t c_sm, int64_t c_sn, const pfk_gemm_epilogue* epi, int* err, void* stream) {
  return guarded([&] {
    PFB_CHECK_ARG(a_hi && b_hi && c, "null pointer");
    pfb::GemmLaunch L;
    L.precision = precision;
    L.a_hi = a_hi; L.a_lo = a_lo; L.b_hi = b_hi; L.b_lo = b_lo;
    L.a_sb = a_sb; L.b_sb = b_sb; L.batch = batch; L.M = M; L.N = N; L.K = K; L.kpad = kpad;
    L.c = c; L.c_sb = c_sb; L.c_sm = c_sm; L.c_sn = c_sn;
    if (epi) {
      L.alpha = epi->alpha;
      L.bias = epi->bias;
      L.act = epi->act;
      L.residual = epi->residual;
      L.r_sb = epi->res_sb; L.r_sm = epi->res_sm; L.r_sn = epi->res_sn;
    }
    L.err = err;
    pfb::launch_gemm(L, as_stream(stream));
  });
}

int pfk_im2col(const float* x, int64_t n, int64_t c, int64_t h, int64_t w, int64_t sn, int64_t sc, int64_t sh,
               int64_t sw, int64_t kh, int64_t kw, int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w,
               int64_t dil_h, int64_t dil_w, int64_t oh, int64_t ow, float* hi, float* lo, uint16_t* bf16,
               int64_t kpad, void* stream) {
  return guarded([&] {
    PFB_CHECK_ARG(x && (hi || bf16), "null pointer");
    pfb::Im2colLaunch L;
    L.x = x; L.n = n; L.c = c; L.h = h; L.w = w; L.sn = sn; L.sc = sc; L.sh = sh; L.sw = sw;
    L.kh = kh; L.kw = kw; L.stride_h = stride_h; L.stride_w = stride_w; L.pad_h = pad_h; L.pad_w = pad_w;
    L.dil_h = dil_h; L.dil_w = dil_w; L.oh = oh; L.ow = ow; L.kpad = kpad;
    if (lo) {
      L.precision = PFC_PRECISION_TF32X3;
      L.hi = hi;
      L.lo = lo;
    } else {
      L.precision = PFC_PRECISION_BF16;
      L.hi = bf16;
    }
    pfb::launch_im2col(L, as_stream(stream));
  });
}

int pfk_pool2d(const float* x, float* y, const pfk_pool_params* p, void* stream) {
  return guarded([&] {
    PFB_CHECK_ARG(x && y && p, "null pointer");
    pfb::PoolLaunch L;
    L.x = x; L.y = y; L.mode = p->mode;
    L.n = p->n; L.c = p->c; L.h = p->h; L.w = p->w; L.sn = p->sn; L.sc = p->sc; L.sh = p->sh; L.sw = p->sw;
    L.kh = p->kh; L.kw = p->kw; L.stride_h = p->stride_h; L.stride_w = p->stride_w; L.pad_h = p->pad_h;
    L.pad_w = p->pad_w; L.oh = p->oh; L.ow = p->ow; L.osn = p->osn; L.osc = p->osc; L.osh = p->osh; L.osw = p->osw;
    pfb::launch_pool(L, as_stream(stream));
  });
}

}  // extern "C"
