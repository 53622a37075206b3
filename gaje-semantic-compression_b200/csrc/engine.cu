// engine.cu -- the B200 decode engine behind include/gaje_cuda.h.
//
// Host side of GenomicLLM for `.gaje.flat` models: load_genomic_auto
// (src/io/flat_reader.rs:240-251) becomes mmap + validate + one device upload
// with the Q4_0 blocks repacked; forward_core (src/nn/llm/forward.rs:7-63)
// becomes one replay of a captured CUDA graph of the step kernels in
// kernels.cuh; generate_native_core (src/nn/llm/forward.rs:215-330) is the
// same host loop around it with the token selection done on the device.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <thread>
#include <mutex>
#include <set>
#include <string>
#include <type_traits>
#include <vector>

#include "flat_format.h"
#include "kernels.cuh"
#include "megakernel.cuh"
#include "gemm.cuh"
#include "batch.cuh"
#include "tc_gemm.cuh"
#include "fused.cuh"
#include "quant.cuh"
#include "sample.cuh"

using namespace gaje;

namespace {

#define CK(expr)                                                                         \
  do {                                                                                   \
    cudaError_t e_ = (expr);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return set_error(GAJE_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---- NCCL, resolved at run time (vocab-sharded serving only).  The library
// does not link libnccl: a host process that already loaded one (a PyTorch
// process, a Rust host with its own NCCL) shares it through the soname, and a
// single-GPU user never needs it.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string why;  // empty when every symbol resolved
};
const NcclApi& nccl_api() {
  static NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      a.why = std::string("libnccl.so.2 could not be loaded: ") + (e ? e : "?");
      return a;
    }
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn && a.why.empty()) a.why = std::string("libnccl lacks ") + name;
    };
    sym(a.get_unique_id, "ncclGetUniqueId");
    sym(a.comm_init_rank, "ncclCommInitRank");
    sym(a.all_gather, "ncclAllGather");
    sym(a.comm_destroy, "ncclCommDestroy");
    sym(a.comm_abort, "ncclCommAbort");
    sym(a.comm_get_async_error, "ncclCommGetAsyncError");
    sym(a.error_string, "ncclGetErrorString");
    return a;
  }();
  return api;
}

// The vocabulary split of the lm_head: rank r owns rows [r*chunk, r*chunk +
// rows) with chunk = ceil(V / nranks).
void vocab_shard(int V, int nranks, int rank, int& row0, int& rows) {
  const int chunk = (V + nranks - 1) / nranks;
  row0 = std::min(V, rank * chunk);
  rows = std::max(0, std::min(chunk, V - row0));
}

// Host twin of the device amax_key: larger value first, then the lower index;
// NaN and -inf never win; -0.0 ties with +0.0.
uint64_t host_amax_key(float v, uint32_t idx) {
  if (!(v > -INFINITY)) return 0ull;
  if (v == 0.0f) v = 0.0f;
  uint32_t u;
  memcpy(&u, &v, 4);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (uint64_t(u) << 32) | (0xFFFFFFFFu - idx);
}

// One device allocation carved into aligned pieces.
struct Arena {
  char* base = nullptr;
  size_t size = 0, used = 0;
  template <class T>
  T* take(size_t count) {
    size_t off = align_up(used, 256);
    used = off + count * sizeof(T);
    return base ? reinterpret_cast<T*>(base + off) : nullptr;
  }
};

struct Q4Dev {
  uint4* qs = nullptr;
  uint32_t* sm = nullptr;
  float* bias = nullptr;
  int N = 0, K = 0, nb = 0, nbp = 0;
  float* lut = nullptr;  // Genomic4Bit centroid tables [N][nb][16] (qs: codes, sm unused)
  // K-block-major copy for the tensor-core GEMM's weight stream (and the fused
  // kernel's column passes): qsT[kb][ldT], smT[kb][ldT], ldT = N rounded up to
  // a multiple of 4; nullptr when the model has no tensor-core path
  uint4* qsT = nullptr;
  uint32_t* smT = nullptr;
  int ldT = 0;
  Q4View view() const { return Q4View{qs, sm, bias, N, K, nb, nbp, lut}; }
  Q4Rows tc_rows() const { return Q4Rows{view(), qsT, smT, ldT}; }
};

constexpr int kMaxDynSmem = 227 * 1024;
constexpr int kBatchMT = 8;  // activation vectors per Q4 GEMM CTA of a batched step
constexpr int kBatchTcMin = 16;  // batch size from which the step's GEMMs run on the tensor cores

// Launch with cudaLaunchKernelEx; `pdl` lets the kernel start before its
// predecessor finishes (programmatic stream serialization): the kernel itself
// calls griddepcontrol.wait before touching its predecessor's outputs.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Work split of one GEMV: units (rows or pairs) per CTA, grid, shared memory.
struct GemvPlan {
  int units = 0, upc = 0, grid = 0;
  size_t smem = 0;
};

GemvPlan plan_gemv(int mode, const Q4Dev& m, int units, int sms) {
  GemvPlan p;
  p.units = units;
  p.upc = (units + sms - 1) / sms;
  const bool lut = m.lut != nullptr;
  while (p.upc > 1 && gemv_smem_bytes(mode, m.K, m.nb, m.nbp, p.upc, lut) > size_t(kMaxDynSmem))
    p.upc = (p.upc + 1) / 2;
  p.grid = (units + p.upc - 1) / p.upc;
  p.smem = gemv_smem_bytes(mode, m.K, m.nb, m.nbp, p.upc, lut);
  return p;
}

// Raises a kernel's dynamic shared-memory limit to at least `bytes` (the
// limit is per function and process-wide, so it only ever grows: a model
// loaded later with a smaller shape must not lower it under an earlier one).
// Any size is raised explicitly, since static shared memory counts against
// the default 48 KB too.
int smem_optin(const void* kern, size_t bytes) {
  if (bytes > size_t(kMaxDynSmem))
    return set_error(GAJE_ERR_UNSUPPORTED, "a kernel needs more than 227 KB of shared memory for this shape");
  static std::mutex mu;
  static std::vector<std::pair<const void*, size_t>> done;
  std::lock_guard<std::mutex> lk(mu);
  int dev = 0;
  cudaGetDevice(&dev);
  const void* key = reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(kern) ^ (uintptr_t(dev) << 56));
  for (auto& kv : done)
    if (kv.first == key && kv.second >= bytes) return GAJE_OK;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
  if (e != cudaSuccess) return set_error(GAJE_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  for (auto& kv : done)
    if (kv.first == key) {
      kv.second = bytes;
      return GAJE_OK;
    }
  done.emplace_back(key, bytes);
  return GAJE_OK;
}

// splitmix64 uniforms in [0,1) with 24 bits, as rand's gen::<f32>() builds them.
struct Rng {
  uint64_t s = 0;
  float uniform() {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return float(uint32_t(z >> 32) >> 8) * (1.0f / 16777216.0f);
  }
};

}  // namespace

// Token selection of generate_native_core on the device, one CTA:
// mode 0 greedy (first max), mode 1 temperature sampling with a host uniform r:
// probs = exp((v - max)/T), choose the first index whose running sum >= r*sum.
__global__ void __launch_bounds__(1024) k_select(const float* logits, int n, int mode, float temperature,
                                                 float r, unsigned* out) {
  __shared__ float redf[32];
  __shared__ unsigned long long redk[32];
  __shared__ float scan[1024];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (mode == 0) {
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const unsigned long long k = amax_key(logits[i], (unsigned)i);
      best = k > best ? k : best;
    }
    best = warp_max_u64(best);
    if (lane == 0) redk[wid] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = 0;
      for (int i = 0; i < nw; ++i) b = redk[i] > b ? redk[i] : b;
      *out = amax_index(b);
    }
    return;
  }
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, logits[i]);
  m = warp_max(m);
  if (lane == 0) redf[wid] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -INFINITY;
    for (int i = 0; i < nw; ++i) b = fmaxf(b, redf[i]);
    redf[0] = b;
  }
  __syncthreads();
  m = redf[0];
  // contiguous chunk per thread, sequential inside the chunk
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int lo = min(n, (int)threadIdx.x * per), hi = min(n, lo + per);
  float local = 0.f;
  for (int i = lo; i < hi; ++i) local += expf((logits[i] - m) / temperature);
  scan[threadIdx.x] = local;
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {  // inclusive Hillis-Steele scan
    const float v = threadIdx.x >= (unsigned)off ? scan[threadIdx.x - off] : 0.f;
    __syncthreads();
    scan[threadIdx.x] += v;
    __syncthreads();
  }
  const float total = scan[blockDim.x - 1];
  const float target = r * total;
  float cum = threadIdx.x ? scan[threadIdx.x - 1] : 0.f;
  if (threadIdx.x == 0) *out = 0u;  // the reference's fallback index
  __syncthreads();
  if (!(target <= scan[threadIdx.x]) || (threadIdx.x && target <= cum)) return;
  for (int i = lo; i < hi; ++i) {
    cum += expf((logits[i] - m) / temperature);
    if (target <= cum) {
      *out = (unsigned)i;
      return;
    }
  }
}

// Repetition penalty of generate_native_core (llm/forward.rs:243-260).
__global__ void k_penalty(float* logits, int n, const unsigned* ids, int n_ids, float p) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_ids; i += gridDim.x * blockDim.x) {
    const unsigned t = ids[i];
    if (t < (unsigned)n) {
      const float v = logits[t];
      logits[t] = v < 0.0f ? v * p : v / p;
    }
  }
}

struct gaje_model {
  int device = 0;
  cudaStream_t stream = nullptr;
  gaje_flat_info info{};
  int d = 0, nh = 0, nkv = 0, hd = 0, ff = 0, V = 0, L = 0, max_ctx = 0, sms = 148;
  // device memory
  Arena arena;
  std::vector<Q4Dev> qkv, wo, gate_up, down;
  std::vector<float*> attn_norm, ffn_norm;
  float* out_norm = nullptr;
  float* embd = nullptr;
  float* lm_head = nullptr;
  float* lm_bias = nullptr;
  float* kcache = nullptr;
  float* vcache = nullptr;
  float2* rope = nullptr;
  float *x = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr;
  float *part_o = nullptr, *part_ml = nullptr;
  unsigned* attn_cnt = nullptr;
  unsigned long long* amax_part = nullptr;
  unsigned* amax_cnt = nullptr;
  unsigned* tok_hist = nullptr;
  unsigned* sel_out = nullptr;
  unsigned* pen_ids = nullptr;
  DevState* st = nullptr;
  // pinned host staging
  DevState* h_st = nullptr;
  unsigned* h_tok = nullptr;
  // step
  StepParams P{};
  GemvPlan pq, po, pg, pd;
  size_t attn_smem = 0;
  int lm_grid = 0, lm_rows = 0, lm_stage_n = 0;
  size_t lm_smem = 0;
  float k_wta_ratio = 0.5f;        // flat_reader.rs:234
  float block_k_wta_ratio = 0.0f;  // block/init.rs:42
  bool use_graph = true;
  cudaGraphExec_t graph = nullptr;
  int graph_kwta_k = -1, graph_block_k = -1;
  uint32_t host_pos = 0;
  Rng rng;
  // persistent decode kernel
  bool use_mega = false;
  MegaPlan mplan{};
  size_t mega_smem = 0;
  LayerW* d_layers = nullptr;
  LLBufs ll{};
  size_t ll_words = 0;
  unsigned epoch = 0;  // LL epochs used so far (the next launch starts after it)
  unsigned long long* phase_ns = nullptr;
  size_t phase_ns_cap = 0;
  unsigned long long* trace_ns = nullptr;
  size_t trace_ns_cap = 0;
  // persistent kernel with two exchanges per block (fused.cuh); preferred
  // over k_decode_mega when the shape fits it
  bool fu_ok = false;      // planned (shape fits, buffers allocated)
  bool use_fused = false;  // planned and launchable
  bool has_lut = false;             // Genomic4Bit tables in the body (kernel-per-phase engine only)
  FusedPlan fplan{};
  int lm_row_bytes = 0;            // bytes of one lm_head row streamed by the fused kernel
  unsigned char* lm_q8 = nullptr;  // fused kernel, Q8_0 lm_head: [Vl][lm_row_bytes] int8 codes, f16 scales
  size_t fused_smem = 0;
  std::vector<FuLayer> h_fl;
  FuLayer* d_fl = nullptr;
  float* fya = nullptr;    // [2][d]
  float* fyb = nullptr;    // [2][d]
  uint2* fwords = nullptr; // phase counters [2 u32] (in a [2][grid] region), kvnew [2][nkv][hd], mlx [nh][S][2], token
  size_t fwords_n = 0;
  unsigned fepoch = 0;
  int withhold_cta = -1;   // gaje_cuda_debug_withhold_flag: for the next fused launch only
  // batched streams (gaje_cuda_forward_batch)
  int max_streams = 0;
  BatchCache bcache{};
  float *bx = nullptr, *bq = nullptr, *battn = nullptr, *bact = nullptr, *blogits = nullptr;
  float *bpart_o = nullptr, *bpart_ml = nullptr;
  unsigned* bcnt = nullptr;
  unsigned long long* blm_part = nullptr;
  unsigned* blm_cnt = nullptr;
  unsigned char* btc_hi = nullptr;  // tensor-core GEMM split activation planes (B >= 16)
  unsigned char* btc_lo = nullptr;
  float* btc_part = nullptr;        // tensor-core split-K partials
  int btc_mpad = 0;                 // rows the planes hold
  float* bsk_part = nullptr;   // Q4 GEMM split partials
  unsigned* bsk_cnt = nullptr; // Q4 GEMM split counters
  size_t bsk_tiles = 0;
  int bsk_per_sm = 1;          // resident Q4 GEMM CTAs per SM
  unsigned* bdev = nullptr;   // [3][max_streams]: tokens, positions, stream ids; then [max_streams] argmax
  unsigned* h_bdev = nullptr; // pinned staging of the same
  std::vector<uint32_t> bpos; // per-stream cache length (host)
  std::vector<cudaGraphExec_t> bgraphs;  // [max_streams + 1]: the captured step per batch size
  int pf_rows = 0;                       // rows of one prefill pass (gaje_load_opts.max_prefill)
  unsigned* pf_tab = nullptr;            // [3][pf_rows]: tokens, positions, stream ids of a prefill chunk
  unsigned* h_pf_tab = nullptr;          // pinned staging of the same
  int blm_grid = 0;                      // lm_head CTAs of a batched step
  // vocab-sharded serving (gaje_cuda_load_sharded): the lm_head holds rows
  // [v0, v0 + Vl) of the vocabulary; Vl == V and nranks == 1 otherwise
  int nranks = 1, rank = 0, v0 = 0, Vl = 0;
  ncclComm_t nccl = nullptr;
  bool nccl_broken = false;              // a collective failed or timed out: the group is gone
  float* bxg = nullptr;                  // [nranks * max_streams][d] residual rows of every rank
  unsigned long long* bkey = nullptr;    // [nranks * max_streams] this rank's best key per gathered row
  unsigned long long* bkey_all = nullptr;  // [nranks][nranks * max_streams]
  // segment timers of the sharded step (events on the model stream): body,
  // residual all-gather, norm + lm_head slice + row argmax, key all-gather +
  // merge; accumulated over the calls since the last gaje_cuda_shard_timings
  cudaEvent_t tev[5] = {};
  double tacc[4] = {0, 0, 0, 0};
  unsigned tcount = 0;

  ~gaje_model() {
    for (cudaEvent_t e : tev)
      if (e) cudaEventDestroy(e);
    if (nccl) {
      const NcclApi& api = nccl_api();
      if (nccl_broken ? api.comm_abort : api.comm_destroy) (nccl_broken ? api.comm_abort : api.comm_destroy)(nccl);
    }
    if (phase_ns) cudaFree(phase_ns);
    if (trace_ns) cudaFree(trace_ns);
    if (graph) cudaGraphExecDestroy(graph);
    for (cudaGraphExec_t g : bgraphs)
      if (g) cudaGraphExecDestroy(g);
    if (arena.base) cudaFree(arena.base);
    if (h_st) cudaFreeHost(h_st);
    if (h_tok) cudaFreeHost(h_tok);
    if (h_bdev) cudaFreeHost(h_bdev);
    if (h_pf_tab) cudaFreeHost(h_pf_tab);
    if (stream) cudaStreamDestroy(stream);
  }

  int logits_k() const {
    if (k_wta_ratio > 0.0f && k_wta_ratio < 1.0f) {
      float kf = float(V) * k_wta_ratio;  // (len as f32 * ratio) as usize, max 1
      return std::max(1, int(kf));
    }
    return 0;
  }
  int block_k() const {
    if (block_k_wta_ratio > 0.0f && block_k_wta_ratio < 1.0f) {
      float kf = float(d) * block_k_wta_ratio;
      return std::max(1, int(kf));
    }
    return 0;
  }

  LayerW layer(int l) const {
    LayerW w;
    w.qkv = qkv[l].view();
    w.wo = wo[l].view();
    w.gate_up = gate_up[l].view();
    w.down = down[l].view();
    w.attn_norm = attn_norm[l];
    w.ffn_norm = ffn_norm[l];
    w.kc = kcache + (size_t)l * nkv * max_ctx * hd;
    w.vc = vcache + (size_t)l * nkv * max_ctx * hd;
    return w;
  }

  AttnArgs attn_args(const LayerW& w) const {
    AttnArgs a;
    a.q = q;
    a.kc = w.kc;
    a.vc = w.vc;
    a.out = attn;
    a.part_o = part_o;
    a.part_ml = part_ml;
    a.cnt = attn_cnt;
    a.bad = nullptr;  // a timeout is reported through st
    a.ctx = 0;
    a.stride = max_ctx;
    a.nh = nh;
    a.nkv = nkv;
    a.hd = hd;
    a.scale = P.attn_scale;
    a.st = st;
    a.fresh = 0;
    return a;
  }

  LmArgs lm_args() const {
    LmArgs a;
    a.W = lm_head;
    a.bias = lm_bias;
    a.flush = P.lm_flush;
    a.x = x;
    a.norm_w = out_norm;
    a.eps = P.eps;
    a.logits = logits;
    a.N = V;
    a.K = d;
    a.rows_per_cta = lm_rows;
    a.stages = lm_stage_n;
    a.part = amax_part;
    a.cnt = amax_cnt;
    a.result = &st->argmax;
    a.st = st;
    a.tok_hist = tok_hist;
    a.hist_cap = unsigned(max_ctx);
    return a;
  }

  // The step's kernel sequence on `stream` (captured once into the graph).
  // Every kernel but the step's first and the K-WTA ones is a PDL launch.
  // With `prof_ms`, every launch is bracketed by events and its time added to
  // prof_ms[class] (profiling only; never captured).
  int launch_step(int kk, int bk, float* prof_ms = nullptr, uint32_t* prof_n = nullptr) {
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (prof_ms) {
      CK(cudaEventCreate(&e0));
      CK(cudaEventCreate(&e1));
    }
    int status = GAJE_OK;
    auto run = [&](int cls, cudaError_t (*fn)(gaje_model*, int, bool), int l, bool pdl) {
      if (status) return;
      if (prof_ms) cudaEventRecord(e0, stream);
      cudaError_t e = fn(this, l, pdl && !prof_ms);
      if (e != cudaSuccess) {
        status = set_error(GAJE_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
        return;
      }
      if (prof_ms) {
        cudaEventRecord(e1, stream);
        cudaEventSynchronize(e1);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        prof_ms[cls] += ms;
        if (prof_n) prof_n[cls] += 1;
      }
    };
    for (int l = 0; l < L; ++l) {
      run(GAJE_K_QKV, &gaje_model::launch_qkv, l, l != 0);
      run(GAJE_K_ATTN, &gaje_model::launch_attn, l, true);
      run(GAJE_K_OPROJ, &gaje_model::launch_oproj, l, true);
      run(GAJE_K_GATEUP, &gaje_model::launch_gateup, l, true);
      run(GAJE_K_DOWN, &gaje_model::launch_down, l, true);
      if (bk > 0) run(GAJE_K_KWTA, &gaje_model::launch_block_kwta, bk, false);
    }
    run(GAJE_K_LMHEAD, &gaje_model::launch_lm, 0, true);
    if (kk > 0) run(GAJE_K_KWTA, &gaje_model::launch_logit_kwta, kk, false);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    return status;
  }

  static cudaError_t launch_qkv(gaje_model* m, int l, bool pdl) {
    GemvArgs a{m->qkv[l].view(), m->pq.units, m->pq.upc, nullptr, nullptr, l};
    return launch_k(k_gemv<G_QKV>, dim3(m->pq.grid), dim3(kGemvThreads), m->pq.smem, m->stream, pdl, m->P,
                    m->layer(l), a);
  }
  static cudaError_t launch_attn(gaje_model* m, int l, bool pdl) {
    return launch_k(k_attn, dim3(m->nkv, kAttnMaxSplits), dim3(kAttnThreads), m->attn_smem, m->stream, pdl,
                    m->attn_args(m->layer(l)));
  }
  static cudaError_t launch_oproj(gaje_model* m, int l, bool pdl) {
    GemvArgs a{m->wo[l].view(), m->po.units, m->po.upc, nullptr, nullptr, l};
    return launch_k(k_gemv<G_OPROJ>, dim3(m->po.grid), dim3(kGemvThreads), m->po.smem, m->stream, pdl, m->P,
                    m->layer(l), a);
  }
  static cudaError_t launch_gateup(gaje_model* m, int l, bool pdl) {
    GemvArgs a{m->gate_up[l].view(), m->pg.units, m->pg.upc, nullptr, nullptr, l};
    return launch_k(k_gemv<G_GATEUP>, dim3(m->pg.grid), dim3(kGemvThreads), m->pg.smem, m->stream, pdl, m->P,
                    m->layer(l), a);
  }
  static cudaError_t launch_down(gaje_model* m, int l, bool pdl) {
    GemvArgs a{m->down[l].view(), m->pd.units, m->pd.upc, nullptr, nullptr, l};
    return launch_k(k_gemv<G_DOWN>, dim3(m->pd.grid), dim3(kGemvThreads), m->pd.smem, m->stream, pdl, m->P,
                    m->layer(l), a);
  }
  static cudaError_t launch_lm(gaje_model* m, int, bool pdl) {
    return launch_k(k_lmhead, dim3(m->lm_grid), dim3(kLmThreads), m->lm_smem, m->stream, pdl, m->lm_args());
  }
  static cudaError_t launch_block_kwta(gaje_model* m, int k, bool) {
    k_kwta<<<1, kKwtaThreads, 0, m->stream>>>(m->x, m->d, k);
    return cudaGetLastError();
  }
  static cudaError_t launch_logit_kwta(gaje_model* m, int k, bool) {
    k_kwta<<<1, kKwtaThreads, 0, m->stream>>>(m->logits, m->V, k);
    return cudaGetLastError();
  }

  // n consecutive greedy steps, each fed the previous step's argmax (the first
  // one fed DevState::token).  With the persistent kernel this is one launch.
  // `trace` (every CTA's in-phase stamps) is only taken when n fits one launch.
  int run_steps(size_t n, unsigned long long* stamps = nullptr, unsigned long long* trace = nullptr) {
    if (n == 0) return GAJE_OK;
    if (use_fused && block_k() == 0 && !stamps && !trace) return run_fused(n);
    if (!use_mega) {
      for (size_t i = 0; i < n; ++i)
        if (int s = run_step()) return s;
      return GAJE_OK;
    }
    while (n > 0) {
      const int chunk = int(std::min<size_t>(n, 1u << 16));
      const unsigned long long per = (unsigned long long)chunk * unsigned(5 * L + 1);
      if ((unsigned long long)epoch + per >= 0xFFFFFFF0ull) {  // epochs wrap: restart from clean words
        CK(cudaMemsetAsync(ll.xa, 0, ll_words * sizeof(uint2), stream));
        epoch = 0;
      }
      MegaArgs a;
      a.P = P;
      a.layers = d_layers;
      a.plan = mplan;
      a.ll = ll;
      a.epoch0 = epoch;
      a.n_steps = chunk;
      a.block_k = block_k();
      a.phase_ns = stamps;
      a.trace_ns = chunk == int(n) ? trace : nullptr;
      epoch += unsigned(per);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(sms);
      cfg.blockDim = dim3(kMkThreads);
      cfg.dynamicSmemBytes = mega_smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      CK(cudaLaunchKernelEx(&cfg, k_decode_mega, a));
      n -= size_t(chunk);
      if (stamps) stamps += size_t(chunk) * (5 * L + 1);
    }
    const int kk = logits_k();
    if (kk > 0) {  // masks the returned logits; the argmax is unaffected
      k_kwta<<<1, kKwtaThreads, 0, stream>>>(logits, V, kk);
      CK(cudaGetLastError());
    }
    return GAJE_OK;
  }

  // n greedy steps in launches of the two-exchange persistent kernel.
  int run_fused(size_t n, unsigned long long* trace = nullptr) {
    // a launch's phase counters reach (steps * L) * grid: keep that below 2^32
    const size_t max_chunk = std::min<size_t>(size_t(1) << 16, (size_t(0xFFFFFFFFu) / (size_t(sms) * L)) - 1);
    while (n > 0) {
      const int chunk = int(std::min<size_t>(n, max_chunk));
      const unsigned long long per = (unsigned long long)chunk * unsigned(2 * L + 1);
      if ((unsigned long long)fepoch + per >= 0xFFFFFFF0ull) {  // epochs wrap: restart from clean words
        CK(cudaMemsetAsync(fwords, 0, fwords_n * sizeof(uint2), stream));
        fepoch = 0;
      }
      CK(cudaMemsetAsync(fya, 0, size_t(4) * d * sizeof(float), stream));  // fya and fyb are adjacent
      CK(cudaMemsetAsync(fwords, 0, 2 * sizeof(unsigned), stream));        // the phase counters
      FusedArgs a;
      a.P = P;
      a.layers = d_layers;
      a.fl = d_fl;
      a.plan = fplan;
      a.ya = fya;
      a.yb = fyb;
      a.cnt = reinterpret_cast<unsigned*>(fwords);
      a.kvnew = fwords + 2 * size_t(sms);
      a.mlx = a.kvnew + 2 * size_t(nkv) * hd;
      a.tok = a.mlx + size_t(nh) * fplan.S * 2;
      a.epoch0 = fepoch;
      a.n_steps = chunk;
      a.trace = chunk == int(n) ? trace : nullptr;
      a.withhold = withhold_cta;
      withhold_cta = -1;
      fepoch += unsigned(per);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(sms);
      cfg.blockDim = dim3(kFuThreads);
      cfg.dynamicSmemBytes = fused_smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      CK(cudaLaunchKernelEx(&cfg, fused_kernel(hd, a.trace != nullptr), a));
      n -= size_t(chunk);
    }
    const int kk = logits_k();
    if (kk > 0) {  // masks the returned logits; the argmax is unaffected
      k_kwta<<<1, kKwtaThreads, 0, stream>>>(logits, V, kk);
      CK(cudaGetLastError());
    }
    return GAJE_OK;
  }

  int run_step() {
    const int kk = logits_k(), bk = block_k();
    if (!use_graph) return launch_step(kk, bk);
    if (!graph || kk != graph_kwta_k || bk != graph_block_k) {
      if (graph) {
        cudaGraphExecDestroy(graph);
        graph = nullptr;
      }
      cudaGraph_t g = nullptr;
      CK(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
      int s = launch_step(kk, bk);
      cudaError_t e = cudaStreamEndCapture(stream, &g);
      if (s) {
        if (g) cudaGraphDestroy(g);
        return s;
      }
      if (e != cudaSuccess) return set_error(GAJE_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
      e = cudaGraphInstantiate(&graph, g, 0);
      cudaGraphDestroy(g);
      if (e != cudaSuccess) {
        graph = nullptr;
        return set_error(GAJE_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
      }
      graph_kwta_k = kk;
      graph_block_k = bk;
    }
    CK(cudaGraphLaunch(graph, stream));
    return GAJE_OK;
  }

  // Reads the device state after a synchronised step: a timed-out bounded wait
  // becomes GAJE_ERR_TIMEOUT, a NaN guard the reference's error string.
  int check_state() {
    if (h_st->err) {
      static const char* kid[] = {"qkv", "oproj", "gateup", "down", "gemv", "", "", "", "attention", "lm_head",
                                  "decode (exchange word)", "decode (producer)", "decode (weight slot)",
                                  "decode (exchange vector)", "decode (publication flag)"};
      const unsigned k = h_st->err - 1;
      std::string m = std::string("a bounded device wait ran out in the ") + (k < 15 ? kid[k] : "?") + " kernel";
      h_st->err = 0;
      cudaMemcpyAsync(&st->err, &h_st->err, 4, cudaMemcpyHostToDevice, stream);
      cudaStreamSynchronize(stream);
      return set_error(GAJE_ERR_TIMEOUT, m);
    }
    if (h_st->nan_code == 0xFFFFFFFFu) return GAJE_OK;
    const unsigned code = h_st->nan_code & 4095u;
    static const char* msgs[] = {"Input x is NaN", "NaN after attn rms_norm", "NaN in up",
                                 "NaN in ffn_out", "NaN in projected_ffn",
                                 "NaN after projected_ffn addition"};
    const unsigned check = code & 7u, layer = code >> 3;
    std::string m = check < 6 ? msgs[check] : "NaN";
    m += " (block " + std::to_string(layer) + ", position " + std::to_string(h_st->nan_code >> 12) + ")";
    h_st->nan_code = 0xFFFFFFFFu;  // re-arm the guard word
    cudaMemcpyAsync(&st->nan_code, &h_st->nan_code, 4, cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
    return set_error(GAJE_ERR_NAN, m);
  }

  int set_pos(uint32_t p) {
    host_pos = p;
    h_st->pos = p;
    CK(cudaMemcpyAsync(&st->pos, &h_st->pos, 4, cudaMemcpyHostToDevice, stream));
    return GAJE_OK;
  }
};

namespace {

// Uploads one engine matrix: its file parts are copied back to back into the
// staging buffer (raw 20-byte blocks, rows in file order), then repacked into
// qs/sm with the row permutation `mode` (see repack_src_row).  The bias is
// concatenated (zero where a part has none) and permuted the same way.
int upload_q4(gaje_model* m, const FlatFile& f, const MatrixRef& ref, Q4Dev& dst, uint32_t* staging, int mode) {
  size_t off = 0;
  for (const FlatEntry* e : ref.parts) {
    CK(cudaMemcpyAsync(reinterpret_cast<char*>(staging) + off, f.blob(e->dna_off, e->dna_len), e->dna_len,
                       cudaMemcpyHostToDevice, m->stream));
    off += e->dna_len;
  }
  CK(cudaMemsetAsync(dst.sm, 0, size_t(dst.N) * dst.nbp * 4, m->stream));
  const size_t nblk = size_t(dst.N) * dst.nb;
  const int blocks = int(std::min<size_t>((nblk + 255) / 256, 8192));
  k_repack_q4<<<blocks, 256, 0, m->stream>>>(staging, dst.N, dst.nb, dst.nbp, mode, m->hd, dst.N / 2, dst.qs, dst.sm);
  CK(cudaGetLastError());
  if (dst.bias) {
    std::vector<float> cat, perm(dst.N, 0.0f);
    for (const FlatEntry* e : ref.parts) {
      std::vector<float> b(e->out, 0.0f);
      if (e->bias_len) memcpy(b.data(), f.blob(e->bias_off, e->bias_len), e->bias_len);
      cat.insert(cat.end(), b.begin(), b.end());
    }
    for (int r = 0; r < dst.N; ++r) perm[r] = cat[repack_src_row(mode, r, m->hd, dst.N / 2)];
    CK(cudaMemcpyAsync(dst.bias, perm.data(), size_t(dst.N) * 4, cudaMemcpyHostToDevice, m->stream));
  }
  CK(cudaStreamSynchronize(m->stream));  // staging and host temporaries are reused
  return GAJE_OK;
}

// Genomic4Bit rows as the engine keeps them (GenomicLinear::new,
// init.rs:29-38 and :109-124): the code of element 2k, stored in the HIGH
// nibble of byte k in the file, moves to the low nibble (the Q4_0 order the
// kernels read), and the centroid table -- 16 floats for the whole matrix,
// 16 per block column, or 16 per (row, block) -- is expanded to one table
// per (row, block).  Rows take the permutation `mode`, as upload_q4's do.
void lut4_rows_host(const uint8_t* nib, const float* cents, size_t n_cents, int N, int K, int mode, int hd,
                    std::vector<uint32_t>& qs_words, std::vector<float>& lut) {
  const size_t nb = size_t(K) / 32;
  qs_words.assign(size_t(N) * nb * 4, 0u);
  lut.assign(size_t(N) * nb * 16, 0.0f);
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)N; ++r) {
    const size_t src = size_t(repack_src_row(mode, int(r), hd, N / 2));
    for (size_t b = 0; b < nb; ++b) {
      uint8_t bytes[16];
      for (int k = 0; k < 16; ++k) {
        const uint8_t v = nib[(src * nb + b) * 16 + k];
        bytes[k] = uint8_t((v >> 4) | (v << 4));
      }
      memcpy(&qs_words[(size_t(r) * nb + b) * 4], bytes, 16);
      const float* c = n_cents == 16 ? cents : n_cents == nb * 16 ? cents + b * 16 : cents + (src * nb + b) * 16;
      memcpy(&lut[(size_t(r) * nb + b) * 16], c, 64);
    }
  }
}

int upload_lut4(gaje_model* m, const FlatFile& f, const MatrixRef& ref, Q4Dev& dst, int mode) {
  const FlatEntry* e = ref.parts[0];  // tables are never split (FlatFile::resolve)
  std::vector<uint32_t> words;
  std::vector<float> lut;
  const float* cents = reinterpret_cast<const float*>(f.blob(e->c_off, e->c_len));
  std::vector<float> cbuf(e->c_len / 4);
  memcpy(cbuf.data(), cents, e->c_len);  // the blob is 64-byte aligned in the file, copied to be safe
  lut4_rows_host(f.blob(e->dna_off, e->dna_len), cbuf.data(), cbuf.size(), dst.N, dst.K, mode, m->hd, words, lut);
  CK(cudaMemcpy(dst.qs, words.data(), words.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dst.lut, lut.data(), lut.size() * 4, cudaMemcpyHostToDevice));
  if (dst.bias) {
    std::vector<float> b(dst.N, 0.0f), perm(dst.N, 0.0f);
    if (e->bias_len) memcpy(b.data(), f.blob(e->bias_off, e->bias_len), e->bias_len);
    for (int r = 0; r < dst.N; ++r) perm[r] = b[repack_src_row(mode, r, m->hd, dst.N / 2)];
    CK(cudaMemcpy(dst.bias, perm.data(), size_t(dst.N) * 4, cudaMemcpyHostToDevice));
  }
  return GAJE_OK;
}

int upload_matrix(gaje_model* m, const FlatFile& f, const MatrixRef& ref, Q4Dev& dst, uint32_t* staging, int mode) {
  return ref.lut ? upload_lut4(m, f, ref, dst, mode) : upload_q4(m, f, ref, dst, staging, mode);
}

// Host libm RoPE table (attention.rs:62-84): freq = 1/powf(base, 2i/hd),
// theta = pos*freq, (cosf, sinf) -- the same glibc calls Rust std makes.
std::vector<float2> rope_table(int max_ctx, int hd, float base) {
  const int half = hd / 2;
  std::vector<float2> t(size_t(max_ctx) * half);
  std::vector<float> freq(half);
  for (int i = 0; i < half; ++i) {
    volatile float e = (2.0f * float(i)) / float(hd);
    volatile float p = powf(base, e);
    freq[i] = 1.0f / p;
  }
  for (int pos = 0; pos < max_ctx; ++pos)
    for (int i = 0; i < half; ++i) {
      volatile float th = float(pos) * freq[i];
      t[size_t(pos) * half + i] = make_float2(cosf(th), sinf(th));
    }
  return t;
}

// Slot ring and work split of the persistent kernel; false when the shape does
// not fit (the kernel-per-phase engine is used instead).
bool plan_mega(gaje_model* m) {
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, k_decode_mega) != cudaSuccess) return false;
  const int G = m->nh / m->nkv;
  const int qd = m->nh * m->hd;
  const int xs = (std::max({m->d, qd, m->ff}) + 31) / 32 * 32;
  if (m->d > kMkMaxNormVec * kMkConsumers || qd != m->d) return false;
  // the split combine keeps kMkCombineElems attention outputs per consumer thread
  if (qd > kMkCombineElems * kMkConsumers) return false;
  MegaPlan& p = m->mplan;
  p.xs_floats = xs;
  if (m->nkv > m->sms) return false;  // one (head, split) unit per CTA at least
  if (m->hd % 32 != 0) return false;  // attention rows are read in whole warps
  p.max_splits = mk_split_cap(m->nkv, m->sms);
  p.attn_chunk_cap = mk_chunk_cap(m->max_ctx, p.max_splits);
  p.ps_floats = (G * p.attn_chunk_cap + 31) / 32 * 32;
  p.qbuf_floats = G * m->hd;
  p.layers_bytes = int((size_t(m->L) * sizeof(LayerW) + 15) / 16 * 16);
  {  // the most bias rows one CTA holds in one GEMV phase
    auto rows = [&](int units, int rpu) { return (units + m->sms - 1) / m->sms * rpu; };
    const int r = std::max({rows(m->qkv[0].N / 2, 2), rows(m->wo[0].N, 1), rows(m->gate_up[0].N / 2, 2),
                            rows(m->down[0].N, 1)});
    p.bias_floats = (r + 31) / 32 * 32;
  }
  const size_t budget = size_t(kMaxDynSmem) - fa.sharedSizeBytes - 1024;
  p.nslots = 0;
  p.slot_bytes = 0;
  const size_t base = mega_smem_bytes(p, m->d, m->hd);
  if (base >= budget) return false;
  auto unit_bytes = [](const Q4Dev& q, int rpu) { return size_t(rpu) * (size_t(q.nb) * 16 + size_t(q.nbp) * 4); };
  const size_t need = std::max({unit_bytes(m->qkv[0], 2), unit_bytes(m->wo[0], 1), unit_bytes(m->gate_up[0], 2),
                                unit_bytes(m->down[0], 1), size_t(m->d) * 4});
  int nslots = int(std::min<size_t>(6, (budget - base) / need));
  if (nslots < 2) return false;
  p.nslots = nslots;
  p.slot_bytes = unsigned((budget - base) / nslots / 128 * 128);
  auto split = [&](MkGemv& g, const Q4Dev& q, int units, int rpu) {
    g.units = units;
    g.upc = (units + m->sms - 1) / m->sms;
    const int fit = int(p.slot_bytes / unit_bytes(q, rpu));
    g.units_per_item = std::max(1, std::min({g.upc, fit, 512 / rpu}));
  };
  split(p.q, m->qkv[0], m->qkv[0].N / 2, 2);
  split(p.o, m->wo[0], m->wo[0].N, 1);
  split(p.g, m->gate_up[0], m->gate_up[0].N / 2, 2);
  split(p.d, m->down[0], m->down[0].N, 1);
  p.lm_rows_per_cta = (m->V + m->sms - 1) / m->sms;
  p.lm_stage_rows = int(std::min<size_t>(kMkConsumerWarps, p.slot_bytes / (size_t(m->d) * 4)));
  m->mega_smem = mega_smem_bytes(p, m->d, m->hd);
  return p.lm_stage_rows >= 1 && m->mega_smem + fa.sharedSizeBytes <= size_t(kMaxDynSmem);
}

// The two-exchange persistent kernel's plan (fused.cuh), from the shapes
// alone; false when the model does not fit it (the five-exchange kernel runs).
// Bytes of one Q8_0 lm_head row as the fused kernel streams it: int8 codes,
// then the f16 scales of its 32-blocks, padded to 16 bytes (bulk copies).
int q8_row_bytes(int d) { return (d + 2 * (d / 32) + 15) / 16 * 16; }

bool plan_fused(gaje_model* m) {
  cudaFuncAttributes fa{};
  const int d = m->d, hd = m->hd, G = m->sms;
  if (d % 32 || (hd != 32 && hd != 64 && hd != 128) || m->ff % 32 || m->info.use_genomic_norm) return false;
  cudaFuncAttributes ft{};
  if (cudaFuncGetAttributes(&fa, fused_kernel(hd, false)) != cudaSuccess ||
      cudaFuncGetAttributes(&ft, fused_kernel(hd, true)) != cudaSuccess)
    return false;
  fa.sharedSizeBytes = std::max(fa.sharedSizeBytes, ft.sharedSizeBytes);
  if (m->qkv[0].K != d || m->gate_up[0].K != d || m->wo[0].N != d || m->down[0].N != d) return false;
  if (m->wo[0].K != m->nh * hd || m->down[0].K != m->ff) return false;
  FusedPlan& p = m->fplan;
  const int s_cta = (G - 2 * m->nkv) / m->nh;
  if (s_cta < 1) return false;
  const int cached = std::max(1, m->max_ctx - 1);
  // splits of ~48 cached positions, plus the one that takes this position's row
  p.S = std::min({s_cta, kFuMaxSplits, std::max(1, (cached + 47) / 48 + 1)});
  p.nA = m->nh * p.S;
  // the k/v rows of this position on as many CTAs as are left (the last
  // splits wait for them), up to 8 per head, an even row count each
  p.kv_split = 1;
  while (p.kv_split < 8 && p.nA + 2 * m->nkv * 2 * p.kv_split <= G && (hd / (2 * p.kv_split)) % 2 == 0)
    p.kv_split *= 2;
  p.nKV = 2 * m->nkv * p.kv_split;
  p.cap = (cached + std::max(1, p.S - 1) - 1) / std::max(1, p.S - 1) + 1;  // fu_split's largest chunk + this row
  p.pv_groups = std::max(1, kFuConsumers / hd);
  p.ob_max = 0;
  p.cb_max = 1;
  for (int c = 0; c < G; ++c) {
    int u0 = 0, n = 0;
    fu_outs(m->ff, G, c, u0, n);
    p.ob_max = std::max(p.ob_max, n);
    if (n > 0) p.cb_max = std::max(p.cb_max, (u0 + n - 1) / 32 - u0 / 32 + 1);
  }
  if (2 * p.ob_max > kFuConsumers || p.cb_max > kFuConsumerWarps) return false;
  p.lm_rows_per_cta = (m->V + G - 1) / G;
  const size_t nbq = size_t(m->qkv[0].nb), nbpq = size_t(m->qkv[0].nbp);
  const size_t nbg = size_t(m->gate_up[0].nb), nbpg = size_t(m->gate_up[0].nbp);
  const size_t need = std::max({size_t(hd) * (nbq * 16 + nbpq * 4), size_t(hd / 32) * d * 20,
                                size_t(2 * p.ob_max) * (nbg * 16 + nbpg * 4), size_t(p.cb_max) * d * 20,
                                size_t(d) * 4});
  p.slot_bytes = unsigned((need + 127) / 128 * 128);
  p.nslots = 0;
  const size_t budget = size_t(kMaxDynSmem) - fa.sharedSizeBytes - 1024;
  const size_t base = fused_smem_bytes(p, d, hd) + 128;  // + the slots' alignment
  if (base >= budget) return false;
  p.nslots = int(std::min<size_t>(kFuMaxSlots, (budget - base) / p.slot_bytes));
  if (p.nslots < 3) return false;
  m->lm_row_bytes = m->info.lm_head_bit_depth == 8 ? q8_row_bytes(d) : d * 4;
  p.lm_stage_rows = int(std::min<size_t>(kFuConsumerWarps, p.slot_bytes / size_t(m->lm_row_bytes)));

  m->fused_smem = fused_smem_bytes(p, d, hd) + 128;
  return p.lm_stage_rows >= 1;
}

// ---- batched streams (gaje_cuda_forward_batch)


int batch_lm_mb(int B) { return B <= 8 ? 8 : 16; }
// ---- tensor-core GEMM launches (k_tc_split + k_q4_gemm_tc)

// The work split of one tensor-core GEMM: vectors per CTA (the MMA's N), the
// padded vector count, and K split across CTAs when the row x vector tiles
// alone would leave SMs idle (every CTA keeps at least four 32-K stages).
struct TcPlan {
  int nt = 0, mpad = 0, z = 1;
  dim3 grid;
  size_t part_floats = 0, tiles = 0;
};
TcPlan tc_plan(int N, int K, int M, int sms) {
  TcPlan p;
  p.nt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  p.mpad = (M + p.nt - 1) / p.nt * p.nt;
  const int gx = (N + kTcRows - 1) / kTcRows, gy = p.mpad / p.nt, nkt = K / kTcK;
  const int want = sms / std::max(1, gx * gy);
  p.z = std::max(1, std::min(want, nkt / 4));
  p.grid = dim3(unsigned(gx), unsigned(gy), unsigned(p.z));
  p.part_floats = p.z > 1 ? size_t(p.z) * M * N : 0;
  p.tiles = size_t(gx) * gy;
  return p;
}
struct TcBuffers {
  unsigned char* hi = nullptr;  // split activation planes, tc_plane_bytes(mpad, K) each
  unsigned char* lo = nullptr;
  float* part = nullptr;        // z * M * N floats when z > 1
};
struct TcNorm {  // the RMSNorm fused into the split (w == nullptr: none)
  const float* w = nullptr;
  float eps = 0.f;
  DevState* st = nullptr;
  const unsigned* pos = nullptr;
  int layer = 0;
};

template <int NT, class WS, class Epi>
cudaError_t tc_launch_nt(const TcPlan& p, const WS& W, int M, Epi epi, const TcBuffers& b, cudaStream_t s, bool pdl,
                         DevState* st) {
  if (smem_optin((const void*)k_q4_gemm_tc<NT, WS, Epi>, tc_smem_bytes(NT))) return cudaErrorInvalidValue;
  return launch_k(k_q4_gemm_tc<NT, WS, Epi>, p.grid, dim3(kTcThreads), tc_smem_bytes(NT), s, pdl, W,
                  (const unsigned char*)b.hi, (const unsigned char*)b.lo, M, p.mpad, TcSplit{b.part}, epi, st);
}

// x [M][K] f32 -> split planes (RMSNorm'd when nm.w) -> y through `epi`;
// every kernel on stream s (the first a programmatic dependent launch when
// pdl).  WS: Q4Rows or F32Rows.
template <class WS, class Epi>
int tc_gemm_run(const TcPlan& p, const WS& W, const float* x, int M, Epi epi, const TcBuffers& b, cudaStream_t s,
                bool pdl, const TcNorm& nm, DevState* st = nullptr) {
  TcSplitArgs sa{x, M, W.K(), p.mpad, nm.w, nm.eps, b.hi, b.lo, nm.st, nm.pos, nm.layer};
  cudaError_t e = launch_k(k_tc_split, dim3(unsigned(p.mpad)), dim3(kTsThreads), 0, s, pdl, sa);
  if (e == cudaSuccess) {
    switch (p.nt) {
      case 16: e = tc_launch_nt<16>(p, W, M, epi, b, s, true, st); break;
      case 32: e = tc_launch_nt<32>(p, W, M, epi, b, s, true, st); break;
      case 64: e = tc_launch_nt<64>(p, W, M, epi, b, s, true, st); break;
      case 128: e = tc_launch_nt<128>(p, W, M, epi, b, s, true, st); break;
      default: e = tc_launch_nt<256>(p, W, M, epi, b, s, true, st); break;
    }
  }
  if (e == cudaSuccess && p.z > 1) {
    const long items = long(M) * ((W.N() + 1) / 2);
    e = launch_k(k_tc_reduce<Epi>, dim3(unsigned((items + 255) / 256)), dim3(256), 0, s, true,
                 (const float*)b.part, p.z, M, W.N(), W.bias(), epi);
  }
  if (e != cudaSuccess) return set_error(GAJE_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return GAJE_OK;
}

// Attention splits of a batched step of Bi streams, at most: enough (stream,
// KV head, split) CTAs to fill the SMs twice, and never chunks of more than
// kBatchAttnRows cached rows (the shared-memory size below), so that long
// contexts are split only as far as needed and the combine stays short.
constexpr int kBatchAttnRows = 96;
int batch_attn_splits(const gaje_model* m, int Bi) {
  const int by_smem = (m->max_ctx + kBatchAttnRows - 1) / kBatchAttnRows;
  const int by_fill = (2 * m->sms) / (Bi * m->nkv);  // two CTAs per SM at most: no tail wave
  return std::max(1, std::min(kAttnMaxSplits, std::max(by_smem, by_fill)));
}
// The streamed attention kernel (k_attn_batch2) serves head_dim 32/64/128 with
// at most kAbMaxGroup query heads per KV head; its splits hold at most
// kAbMaxChunk positions and fill the SMs twice.
bool batch_attn2(const gaje_model* m) {
  return (m->hd == 32 || m->hd == 64 || m->hd == 128) && m->nh / m->nkv <= kAbMaxGroup;
}
int batch_attn2_splits(const gaje_model* m, int Bi) {
  const int by_len = (m->max_ctx + kAbMaxChunk - 1) / kAbMaxChunk;
  const int by_fill = (2 * m->sms) / (Bi * m->nkv);  // two CTAs per SM at most: no tail wave
  return std::max(1, std::min(kAttnMaxSplits, std::max(by_len, by_fill)));
}
cudaError_t launch_attn2(gaje_model* m, int Bi, const AttnBatchArgs& aa) {
  const dim3 grid(unsigned(m->nkv), unsigned(aa.max_splits), unsigned(Bi));
  const size_t smem = attn_batch2_smem(m->nh / m->nkv, m->hd);
  switch (m->hd) {
    case 32: return launch_k(k_attn_batch2<1>, grid, dim3(kAbThreads), smem, m->stream, true, aa);
    case 64: return launch_k(k_attn_batch2<2>, grid, dim3(kAbThreads), smem, m->stream, true, aa);
    default: return launch_k(k_attn_batch2<4>, grid, dim3(kAbThreads), smem, m->stream, true, aa);
  }
}
size_t batch_attn_smem(const gaje_model* m) {  // the largest chunk any batch size gives
  const int ms = std::min(kAttnMaxSplits, std::max(1, (m->max_ctx + kBatchAttnRows - 1) / kBatchAttnRows));
  return attn_smem_bytes(m->nh / m->nkv, m->hd, attn_chunk_max(m->max_ctx, ms));
}

// Shared-memory opt-ins and the lm_head grid, once at load (never during a
// capture).
int batch_setup(gaje_model* m) {
  const size_t sk = skinny_smem_bytes(kBatchMT);
  if (int e = smem_optin((const void*)k_q4_gemm_skinny<kBatchMT, true, EpiQkvBatch>, sk)) return e;
  if (int e = smem_optin((const void*)k_q4_gemm_skinny<kBatchMT, false, EpiResidBatch>, sk)) return e;
  if (int e = smem_optin((const void*)k_q4_gemm_skinny<kBatchMT, true, EpiSwigluBatch>, sk)) return e;
  if (int e = smem_optin((const void*)k_attn_batch, batch_attn_smem(m))) return e;
  if (batch_attn2(m)) {
    const size_t s2 = attn_batch2_smem(m->nh / m->nkv, m->hd);
    if (int e = smem_optin((const void*)k_attn_batch2<1>, s2)) return e;
    if (int e = smem_optin((const void*)k_attn_batch2<2>, s2)) return e;
    if (int e = smem_optin((const void*)k_attn_batch2<4>, s2)) return e;
  }
  if (m->pf_rows > 0) {
    if (int e = smem_optin((const void*)k_attn_prefill, attn_prefill_smem(m->nh / m->nkv, m->hd))) return e;
    if (m->hd == 64)
      if (int e = smem_optin((const void*)k_attn_prefill_tc<64>, attn_tc_smem(64))) return e;
    if (m->hd == 128)
      if (int e = smem_optin((const void*)k_attn_prefill_tc<128>, attn_tc_smem(128))) return e;
  }
  const size_t lm8 = size_t(8) * m->d * 4, lm16 = size_t(16) * m->d * 4;
  if (int e = smem_optin((const void*)k_lmhead_batch<8, 4>, lm8)) return e;
  if (int e = smem_optin((const void*)k_lmhead_batch<16, 2>, lm16)) return e;
  int per = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_lmhead_batch<16, 2>, kLbThreads, lm16));
  m->blm_grid = m->sms * std::max(1, std::min(per, 4));
  int sk_per = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&sk_per, k_q4_gemm_skinny<kBatchMT, true, EpiSwigluBatch>,
                                                   kSkThreads, sk));
  m->bsk_per_sm = std::max(1, sk_per);
  if (m->btc_hi) {  // every tensor-core instantiation a step may launch (never during a capture)
    int e = 0;
    auto optin_nt = [&](auto nt_tag) {
      constexpr int NT = decltype(nt_tag)::value;
      const size_t b = tc_smem_bytes(NT);
      e = e ? e : smem_optin((const void*)k_q4_gemm_tc<NT, Q4Rows, EpiQkvBatch>, b);
      e = e ? e : smem_optin((const void*)k_q4_gemm_tc<NT, Q4Rows, EpiResidBatch>, b);
      e = e ? e : smem_optin((const void*)k_q4_gemm_tc<NT, Q4Rows, EpiSwigluBatch>, b);
      e = e ? e : smem_optin((const void*)k_q4_gemm_tc<NT, F32Rows, EpiStore>, b);
    };
    optin_nt(std::integral_constant<int, 16>{});
    optin_nt(std::integral_constant<int, 32>{});
    optin_nt(std::integral_constant<int, 64>{});
    optin_nt(std::integral_constant<int, 128>{});
    optin_nt(std::integral_constant<int, 256>{});
    if (e) return e;
  }
  return GAJE_OK;
}

// Grid of one Q4 GEMM of a batched step: K splits across CTAs when K spans
// more than one split, and the fewest row pairs per warp that still fit the
// launch in one wave of resident CTAs.
struct SkLaunch {
  dim3 grid;
  SkSplit sp;
};
SkLaunch sk_plan(const gaje_model* m, const Q4Dev& q, int Bi) {
  SkLaunch r;
  const unsigned mtiles = unsigned((Bi + kBatchMT - 1) / kBatchMT);
  const unsigned z = unsigned((q.K + kSkChunk - 1) / kSkChunk);
  const long slots = long(m->sms) * m->bsk_per_sm;
  int ppw = 1;
  auto gx = [&](int p) { return unsigned((q.N + 2 * kSkWarps * p - 1) / (2 * kSkWarps * p)); };
  while (ppw < 8 && long(gx(ppw)) * mtiles * z > slots) ++ppw;
  r.grid = dim3(gx(ppw), mtiles, z);
  r.sp.ppw = ppw;
  r.sp.part = z > 1 ? m->bsk_part : nullptr;
  r.sp.cnt = z > 1 ? m->bsk_cnt : nullptr;
  return r;
}

// One projection of a batched step: the tensor cores (bf16 hi/lo x3) from
// kBatchTcMin streams on, else the CUDA-core skinny GEMM.  `norm` is the
// RMSNorm fused into the activation staging (w == nullptr: none).
template <bool NORM, class Epi>
cudaError_t batch_gemm(gaje_model* m, int Bi, const Q4Dev& q, const float* x, const TcNorm& norm, Epi epi) {
  if (Bi >= kBatchTcMin && m->btc_hi && q.K % kTcK == 0 && q.qsT) {
    const TcPlan p = tc_plan(q.N, q.K, Bi, m->sms);
    TcBuffers b{m->btc_hi, m->btc_lo, m->btc_part};
    return tc_gemm_run(p, q.tc_rows(), x, Bi, epi, b, m->stream, true, norm, m->st) == GAJE_OK
               ? cudaSuccess
               : cudaErrorLaunchFailure;
  }
  SkNorm sn{norm.w, norm.eps, norm.st, norm.pos, norm.layer};
  SkLaunch pl = sk_plan(m, q, Bi);
  return launch_k(k_q4_gemm_skinny<kBatchMT, NORM, Epi>, pl.grid, dim3(kSkThreads), skinny_smem_bytes(kBatchMT),
                  m->stream, true, q.view(), x, Bi, sn, pl.sp, epi);
}

// The kernels of one batched step for the first Bi entries of the stream
// table (already on the device), in stream order, every launch after the
// first a programmatic dependent launch.  Nothing here depends on the
// streams' positions, so the sequence is captured once per Bi.
// Per-class timing of one eagerly launched batched step (profiling only).
struct StepProf {
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  float ms[GAJE_K_COUNT] = {};
  uint32_t n[GAJE_K_COUNT] = {};
};

int launch_batch(gaje_model* m, int Bi, StepProf* prof = nullptr) {
  cudaStream_t st = m->stream;
  auto t0 = [&]() {
    if (prof) cudaEventRecord(prof->e0, st);
  };
  auto t1 = [&](int cls) {
    if (!prof) return;
    cudaEventRecord(prof->e1, st);
    cudaEventSynchronize(prof->e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, prof->e0, prof->e1);
    prof->ms[cls] += ms;
    prof->n[cls] += 1;
  };
  const size_t S = size_t(m->max_streams);
  BatchStreams bs{m->bdev, m->bdev + S, m->bdev + 2 * S};
  unsigned* d_argmax = m->bdev + 3 * S;
  const int d = m->d, L = m->L;
  const float eps = m->info.eps;
  constexpr int MT = kBatchMT;
  const size_t sk = skinny_smem_bytes(MT);
  const int asplit = batch_attn_splits(m, Bi);
  int ns_max = 1, ch_max = 1;  // attention splits at the longest context
  attn_splits(m->max_ctx, ns_max, ch_max, asplit);
  cudaError_t e = launch_k(k_embed_batch, dim3(Bi), dim3(256), 0, st, false, (const float*)m->embd, m->V, d, bs,
                           m->bx);
  for (int l = 0; l < L && e == cudaSuccess; ++l) {
    EpiQkvBatch eq{m->bq, m->bcache, bs, m->rope, m->nh, m->nkv, m->hd, int(m->info.rope_split), l};
    t0();
    e = batch_gemm<true>(m, Bi, m->qkv[l], m->bx, TcNorm{m->attn_norm[l], eps, m->st, bs.pos, l}, eq);
    t1(GAJE_K_QKV);
    if (e != cudaSuccess) break;
    AttnBatchArgs aa{m->bq, m->battn, m->bcache, bs, m->bpart_o, m->bpart_ml, m->bcnt, l, m->nh,
                     1.0f / sqrtf(float(m->hd)), asplit};
    t0();
    if (batch_attn2(m)) {
      aa.max_splits = batch_attn2_splits(m, Bi);
      e = launch_attn2(m, Bi, aa);
    } else {
      e = launch_k(k_attn_batch, dim3(unsigned(m->nkv), unsigned(ns_max), unsigned(Bi)), dim3(kAttnThreads),
                   batch_attn_smem(m), st, true, aa);
    }
    t1(GAJE_K_ATTN);
    if (e != cudaSuccess) break;
    t0();
    e = batch_gemm<false>(m, Bi, m->wo[l], m->battn, TcNorm{}, EpiResidBatch{m->bx, d, nullptr, bs, l});
    t1(GAJE_K_OPROJ);
    if (e != cudaSuccess) break;
    t0();
    e = batch_gemm<true>(m, Bi, m->gate_up[l], m->bx, TcNorm{m->ffn_norm[l], eps, nullptr, bs.pos, l},
                         EpiSwigluBatch{m->bact, m->ff, m->st, bs, l});
    t1(GAJE_K_GATEUP);
    if (e != cudaSuccess) break;
    t0();
    e = batch_gemm<false>(m, Bi, m->down[l], m->bact, TcNorm{}, EpiResidBatch{m->bx, d, m->st, bs, l});
    t1(GAJE_K_DOWN);
  }
  t0();
  if (m->nranks > 1) {  // vocab-sharded: the head runs after the step graph (sharded_head)
    if (e != cudaSuccess) return set_error(GAJE_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
    return GAJE_OK;
  }
  if (e == cudaSuccess && Bi >= kBatchTcMin && m->btc_hi && d % kTcK == 0) {
    // output norm fused into the split, f32 lm_head on the tensor cores, then the argmax per stream
    const TcPlan p = tc_plan(m->V, d, Bi, m->sms);
    TcBuffers b{m->btc_hi, m->btc_lo, m->btc_part};
    if (tc_gemm_run(p, F32Rows{m->lm_head, m->lm_bias, m->V, d}, m->bx, Bi, EpiStore{m->blogits, m->V}, b, st, true,
                    TcNorm{m->out_norm, eps, nullptr, bs.pos, L}, m->st) != GAJE_OK)
      return set_error(GAJE_ERR_CUDA, "kernel launch: lm_head");
    e = launch_k(k_argmax_rows, dim3(unsigned(Bi)), dim3(512), 0, st, true, (const float*)m->blogits, m->V, d_argmax,
                 0u, (unsigned long long*)nullptr);
    t1(GAJE_K_LMHEAD);
    if (e != cudaSuccess) return set_error(GAJE_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
    return GAJE_OK;
  }
  const int MB = batch_lm_mb(Bi);
  for (int b0 = 0; b0 < Bi && e == cudaSuccess; b0 += MB) {
    LmBatchArgs la{};
    la.W = m->lm_head;
    la.bias = m->lm_bias;
    la.x = m->bx + size_t(b0) * d;
    la.norm_w = m->out_norm;
    la.eps = eps;
    la.logits = m->blogits + size_t(b0) * m->V;
    la.part = m->blm_part;
    la.cnt = m->blm_cnt;
    la.argmax = d_argmax + b0;
    la.V = m->V;
    la.d = d;
    la.B = std::min(MB, Bi - b0);
    la.rows_per_cta = (m->V + m->blm_grid - 1) / m->blm_grid;
    la.flush = m->P.lm_flush;
    const size_t smem = size_t(MB) * d * 4;
    e = MB == 8 ? launch_k(k_lmhead_batch<8, 4>, dim3(m->blm_grid), dim3(kLbThreads), smem, st, true, la)
                : launch_k(k_lmhead_batch<16, 2>, dim3(m->blm_grid), dim3(kLbThreads), smem, st, true, la);
  }
  t1(GAJE_K_LMHEAD);
  if (e != cudaSuccess) return set_error(GAJE_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return GAJE_OK;
}

// One prefill chunk of stream `sid`: rows 0..nc-1 of the prefill table (tokens,
// positions p0.., the stream id) through every block -- whole-chunk GEMMs,
// the k/v rows written into the stream's cache by the QKV epilogue, then the
// causal attention pass -- leaving the residual rows in bx.  With `head`,
// the output norm + lm_head + argmax of the chunk's last row follow.
int launch_prefill_chunk(gaje_model* m, int nc, int p0, unsigned sid, bool head) {
  cudaStream_t st = m->stream;
  const size_t R = size_t(m->pf_rows);
  BatchStreams bs{m->pf_tab, m->pf_tab + R, m->pf_tab + 2 * R};
  const int d = m->d, L = m->L, G = m->nh / m->nkv;
  const float eps = m->info.eps;
  cudaError_t e = launch_k(k_embed_batch, dim3(unsigned(nc)), dim3(256), 0, st, false, (const float*)m->embd, m->V,
                           d, bs, m->bx);
  const int qb = attn_prefill_qb(G);
  for (int l = 0; l < L && e == cudaSuccess; ++l) {
    EpiQkvBatch eq{m->bq, m->bcache, bs, m->rope, m->nh, m->nkv, m->hd, int(m->info.rope_split), l};
    e = batch_gemm<true>(m, nc, m->qkv[l], m->bx, TcNorm{m->attn_norm[l], eps, m->st, bs.pos, l}, eq);
    if (e != cudaSuccess) break;
    AttnPrefillArgs ap{m->bq, m->battn, m->bcache.k + m->bcache.row(sid, l, 0, 0),
                       m->bcache.v + m->bcache.row(sid, l, 0, 0), nc, p0, m->nh, m->nkv, m->hd, m->max_ctx,
                       1.0f / sqrtf(float(m->hd))};
    const dim3 agrid(unsigned((nc + qb - 1) / qb), unsigned(m->nkv));
    if (m->hd == 64)  // tensor cores for the head dims the configs use
      e = launch_k(k_attn_prefill_tc<64>, agrid, dim3(kAtThreads), attn_tc_smem(64), st, true, ap);
    else if (m->hd == 128)
      e = launch_k(k_attn_prefill_tc<128>, agrid, dim3(kAtThreads), attn_tc_smem(128), st, true, ap);
    else
      e = launch_k(k_attn_prefill, agrid, dim3(kApThreads), attn_prefill_smem(G, m->hd), st, true, ap);
    if (e != cudaSuccess) break;
    e = batch_gemm<false>(m, nc, m->wo[l], m->battn, TcNorm{}, EpiResidBatch{m->bx, d, nullptr, bs, l});
    if (e != cudaSuccess) break;
    e = batch_gemm<true>(m, nc, m->gate_up[l], m->bx, TcNorm{m->ffn_norm[l], eps, nullptr, bs.pos, l},
                         EpiSwigluBatch{m->bact, m->ff, m->st, bs, l});
    if (e != cudaSuccess) break;
    e = batch_gemm<false>(m, nc, m->down[l], m->bact, TcNorm{}, EpiResidBatch{m->bx, d, m->st, bs, l});
  }
  if (e == cudaSuccess && head && m->nranks == 1) {
    LmBatchArgs la{};
    la.W = m->lm_head;
    la.bias = m->lm_bias;
    la.x = m->bx + size_t(nc - 1) * d;
    la.norm_w = m->out_norm;
    la.eps = eps;
    la.logits = m->blogits;
    la.part = m->blm_part;
    la.cnt = m->blm_cnt;
    la.argmax = m->bdev + 3 * size_t(m->max_streams);
    la.V = m->V;
    la.d = d;
    la.B = 1;
    la.rows_per_cta = (m->V + m->blm_grid - 1) / m->blm_grid;
    la.flush = m->P.lm_flush;
    e = launch_k(k_lmhead_batch<8, 4>, dim3(m->blm_grid), dim3(kLbThreads), size_t(8) * d * 4, st, true, la);
  }
  if (e != cudaSuccess) return set_error(GAJE_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return GAJE_OK;
}

// ---- the vocab-sharded head of a batched step (gaje_cuda_load_sharded)
//
// Every rank holds the whole body and the lm_head rows [v0, v0 + Vl).  After
// the body of a step (B residual rows of this rank's streams in x_local):
//   1. all-gather the residual rows of every rank      -> bxg [nranks*B][d]
//   2. output norm + this rank's lm_head rows for all nranks*B rows, and per
//      row the best amax_key over those rows (global index) -> bkey
//   3. all-gather the keys                              -> bkey_all [nranks][nranks*B]
//   4. per local stream the largest key over the ranks -> its first-max argmax
// The largest key is the first maximum over the whole vocabulary, as the
// single-GPU argmax (llm/forward.rs:262-271) gives it.  Every rank must issue
// the same sequence of sharded calls with the same B: the two all-gathers
// are collective.
int sharded_head(gaje_model* m, const float* x_local, int B, unsigned* d_argmax) {
  const NcclApi& api = nccl_api();
  cudaStream_t st = m->stream;
  const int d = m->d, n = m->nranks, M = n * B;
  const float eps = m->info.eps;
  auto nccl_fail = [&](ncclResult_t r, const char* what) {
    m->nccl_broken = true;
    return set_error(GAJE_ERR_CUDA, std::string("NCCL ") + what + ": " + api.error_string(r));
  };
  ncclResult_t r = api.all_gather(x_local, m->bxg, size_t(B) * d, ncclFloat32, m->nccl, st);
  if (r != ncclSuccess) return nccl_fail(r, "all-gather of the residual rows");
  if (m->tev[2]) CK(cudaEventRecord(m->tev[2], st));
  cudaError_t e = cudaSuccess;
  if (M >= kBatchTcMin && m->btc_hi && d % kTcK == 0) {
    // output norm fused into the split, this rank's vocab rows on the tensor cores
    const TcPlan p = tc_plan(m->Vl, d, M, m->sms);
    TcBuffers b{m->btc_hi, m->btc_lo, m->btc_part};
    if (tc_gemm_run(p, F32Rows{m->lm_head, m->lm_bias, m->Vl, d}, m->bxg, M, EpiStore{m->blogits, m->Vl}, b, st,
                    false, TcNorm{m->out_norm, eps, nullptr, nullptr, m->L}, m->st) != GAJE_OK)
      return set_error(GAJE_ERR_CUDA, "kernel launch: sharded lm_head");
    e = launch_k(k_argmax_rows, dim3(unsigned(M)), dim3(512), 0, st, true, (const float*)m->blogits, m->Vl,
                 (unsigned*)nullptr, unsigned(m->v0), m->bkey);
  } else {
    const int MB = batch_lm_mb(M);
    for (int b0 = 0; b0 < M && e == cudaSuccess; b0 += MB) {
      LmBatchArgs la{};
      la.W = m->lm_head;
      la.bias = m->lm_bias;
      la.x = m->bxg + size_t(b0) * d;
      la.norm_w = m->out_norm;
      la.eps = eps;
      la.logits = m->blogits + size_t(b0) * m->Vl;
      la.part = m->blm_part;
      la.cnt = m->blm_cnt;
      la.argmax = nullptr;
      la.keys = m->bkey + b0;
      la.row_offset = unsigned(m->v0);
      la.V = m->Vl;
      la.d = d;
      la.B = std::min(MB, M - b0);
      la.rows_per_cta = (m->Vl + m->blm_grid - 1) / m->blm_grid;
      la.flush = m->P.lm_flush;
      const size_t smem = size_t(MB) * d * 4;
      e = MB == 8 ? launch_k(k_lmhead_batch<8, 4>, dim3(m->blm_grid), dim3(kLbThreads), smem, st, false, la)
                  : launch_k(k_lmhead_batch<16, 2>, dim3(m->blm_grid), dim3(kLbThreads), smem, st, false, la);
    }
  }
  if (e != cudaSuccess) return set_error(GAJE_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  if (m->tev[3]) CK(cudaEventRecord(m->tev[3], st));
  r = api.all_gather(m->bkey, m->bkey_all, size_t(M), ncclUint64, m->nccl, st);
  if (r != ncclSuccess) return nccl_fail(r, "all-gather of the argmax keys");
  k_shard_argmax<<<1, 256, 0, st>>>(m->bkey_all, n, B, m->rank, d_argmax);
  CK(cudaGetLastError());
  if (m->tev[4]) CK(cudaEventRecord(m->tev[4], st));
  return GAJE_OK;
}

// Waits for the model stream after a sharded step, bounded: a rank whose peer
// died never sees its collective finish, so after GAJE_NCCL_TIMEOUT_S seconds
// (default 120) the communicator is aborted and the call fails with
// GAJE_ERR_TIMEOUT; the model then refuses further sharded calls.
int sync_sharded(gaje_model* m) {
  const NcclApi& api = nccl_api();
  double limit = 120.0;
  if (const char* s = getenv("GAJE_NCCL_TIMEOUT_S")) limit = std::max(0.1, atof(s));
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(m->stream);
    if (q == cudaSuccess) return GAJE_OK;
    if (q != cudaErrorNotReady) return set_error(GAJE_ERR_CUDA, std::string("step: ") + cudaGetErrorString(q));
    ncclResult_t ae = ncclSuccess;
    if (api.comm_get_async_error(m->nccl, &ae) == ncclSuccess && ae != ncclSuccess && ae != ncclInProgress) {
      m->nccl_broken = true;
      api.comm_abort(m->nccl);
      m->nccl = nullptr;
      return set_error(GAJE_ERR_CUDA, std::string("NCCL: ") + api.error_string(ae));
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit) {
      m->nccl_broken = true;
      api.comm_abort(m->nccl);
      m->nccl = nullptr;
      return set_error(GAJE_ERR_TIMEOUT, "a collective of the sharded step did not finish (a peer rank is gone?)");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

int load_impl(gaje_model* m, const char* path, const gaje_load_opts* opts) {
  FlatFile f;
  std::string err;
  if (int s = f.open(path, err)) return set_error(s, err);
  const gaje_flat_info& I = f.info;
  if ((I.embd_bit_depth != 32 && I.embd_bit_depth != 8) || (I.lm_head_bit_depth != 32 && I.lm_head_bit_depth != 8))
    return set_error(GAJE_ERR_UNSUPPORTED, "token_embd/lm_head must be f32 or Q8_0");
  if (I.n_embd % 32 != 0) return set_error(GAJE_ERR_UNSUPPORTED, "n_embd must be a multiple of 32");
  // Genomic4Bit tables (init.rs:36-37) run on the kernel-per-phase engine,
  // whose GEMV launches are planned once per matrix kind: a kind is a table
  // in every block or in none
  m->has_lut = false;
  for (int k = 0; k < 4 && !f.blocks.empty(); ++k) {
    auto pick = [k](const BlockRefs& b) { return k == 0 ? b.qkv.lut : k == 1 ? b.wo.lut : k == 2 ? b.gate_up.lut : b.down.lut; };
    const bool first = pick(f.blocks[0]);
    for (const BlockRefs& b : f.blocks)
      if (pick(b) != first)
        return set_error(GAJE_ERR_UNSUPPORTED, "a matrix kind mixes Genomic4Bit tables and Q4_0 blocks across blocks");
    m->has_lut |= first;
  }
  if (m->has_lut && opts && (opts->max_streams > 0 || opts->max_prefill > 0))
    return set_error(GAJE_ERR_UNSUPPORTED,
                     "Genomic4Bit tables run on the single-stream engine only (max_streams and max_prefill must be 0)");
  if (m->has_lut && m->nranks > 1)
    return set_error(GAJE_ERR_UNSUPPORTED, "Genomic4Bit tables are not supported by the sharded engine");
  m->info = I;
  m->d = int(I.n_embd);
  m->nh = int(I.n_head);
  m->nkv = int(I.n_head_kv);
  m->hd = int(I.head_dim);
  m->ff = int(I.ffn_dim);
  m->V = int(I.vocab_size);
  m->L = int(I.n_blocks);
  vocab_shard(m->V, m->nranks, m->rank, m->v0, m->Vl);
  m->max_ctx = int(opts && opts->max_ctx ? opts->max_ctx : 4096);
  m->use_graph = !opts || opts->use_graph;
  m->max_streams = opts ? int(opts->max_streams) : 0;
  if (m->max_streams < 0 || m->max_streams > 1024)
    return set_error(GAJE_ERR_INVALID, "max_streams above 1024");
  m->pf_rows = opts ? int(opts->max_prefill) : 0;
  if (m->pf_rows < 0 || m->pf_rows > 65536) return set_error(GAJE_ERR_INVALID, "max_prefill above 65536");
  if (m->pf_rows > 0 && m->max_streams == 0)
    return set_error(GAJE_ERR_INVALID, "max_prefill needs batched streams (max_streams > 0)");
  if (m->pf_rows > 0 && m->hd > 128)
    return set_error(GAJE_ERR_UNSUPPORTED, "prefill attention supports head_dim up to 128");
  if (m->nranks > 1 && m->max_streams == 0)
    return set_error(GAJE_ERR_INVALID, "a vocab-sharded model serves batched streams: set max_streams");
  if (m->Vl < 1) return set_error(GAJE_ERR_INVALID, "more ranks than vocabulary rows");
  m->rng.s = opts ? opts->seed : 0;
  if (m->nh / m->nkv > kAttnMaxGroup) return set_error(GAJE_ERR_UNSUPPORTED, "more than 16 query heads per KV head");
  if (m->hd % 4 != 0) return set_error(GAJE_ERR_UNSUPPORTED, "head_dim must be a multiple of 4");
  if (m->max_ctx > (1 << 20)) return set_error(GAJE_ERR_INVALID, "max_ctx above 2^20");
  CK(cudaSetDevice(m->device));
  CK(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, m->device);
  // ---- plan the arena (sizes only), then allocate and carve for real
  const size_t V = m->V, d = m->d, L = m->L;
  size_t staging_bytes = 0;
  // the batched engine's tensor-core GEMMs (see the btc_* buffers below) and
  // the K-block-major weight copies they stream
  const size_t tc_rows = std::max(std::max(size_t(m->max_streams), size_t(m->pf_rows)),
                                  size_t(m->nranks) * size_t(m->max_streams));
  const bool tc_on = m->max_streams > 0 && tc_rows >= size_t(kBatchTcMin);
  auto plan = [&](Arena& a) {
    m->qkv.assign(L, Q4Dev());
    m->wo.assign(L, Q4Dev());
    m->gate_up.assign(L, Q4Dev());
    m->down.assign(L, Q4Dev());
    m->attn_norm.assign(L, nullptr);
    m->ffn_norm.assign(L, nullptr);
    for (size_t l = 0; l < L; ++l) {
      const BlockRefs& b = f.blocks[l];
      const MatrixRef* refs[4] = {&b.qkv, &b.wo, &b.gate_up, &b.down};
      Q4Dev* dsts[4] = {&m->qkv[l], &m->wo[l], &m->gate_up[l], &m->down[l]};
      for (int k = 0; k < 4; ++k) {
        Q4Dev& q = *dsts[k];
        q.N = int(refs[k]->out);
        q.K = int(refs[k]->in);
        q.nb = q.K / 32;
        q.nbp = (q.nb + 3) / 4 * 4;
        q.qs = a.take<uint4>(size_t(q.N) * q.nb);
        q.sm = refs[k]->lut ? nullptr : a.take<uint32_t>(size_t(q.N) * q.nbp);
        q.lut = refs[k]->lut ? a.take<float>(size_t(q.N) * q.nb * 16) : nullptr;
        q.bias = refs[k]->has_bias ? a.take<float>(q.N) : nullptr;
        if (tc_on && !refs[k]->lut) {  // the tensor-core GEMMs stream this copy
          q.ldT = (q.N + 3) / 4 * 4;
          q.qsT = a.take<uint4>(size_t(q.ldT) * q.nb);
          q.smT = a.take<uint32_t>(size_t(q.ldT) * q.nb);
        }
        size_t tot = 0;
        for (const FlatEntry* e : refs[k]->parts) tot += e->dna_len;
        staging_bytes = std::max(staging_bytes, tot);
      }
      m->attn_norm[l] = a.take<float>(d);
      m->ffn_norm[l] = a.take<float>(d);
    }
    m->out_norm = a.take<float>(d);
    m->embd = a.take<float>(V * d);
    m->lm_head = a.take<float>(size_t(m->Vl) * d);  // this rank's vocab rows (all of them unsharded)
    m->lm_bias = f.lm_head->bias_len ? a.take<float>(size_t(m->Vl)) : nullptr;
    const size_t cache = L * size_t(m->nkv) * m->max_ctx * m->hd;
    m->kcache = a.take<float>(cache);
    m->vcache = a.take<float>(cache);
    m->rope = a.take<float2>(size_t(m->max_ctx) * (m->hd / 2));
    m->x = a.take<float>(d);
    m->q = a.take<float>(size_t(m->nh) * m->hd);
    m->attn = a.take<float>(size_t(m->nh) * m->hd);
    m->act = a.take<float>(m->ff);
    m->logits = a.take<float>(V);
    m->part_o = a.take<float>(size_t(m->nkv) * kAttnMaxSplits * (m->nh / m->nkv) * m->hd);
    m->part_ml = a.take<float>(size_t(m->nkv) * kAttnMaxSplits * (m->nh / m->nkv) * 2);
    m->attn_cnt = a.take<unsigned>(m->nkv);
    m->amax_part = a.take<unsigned long long>(m->sms);
    m->amax_cnt = a.take<unsigned>(1);
    m->tok_hist = a.take<unsigned>(m->max_ctx);
    m->sel_out = a.take<unsigned>(1);
    m->pen_ids = a.take<unsigned>(m->max_ctx);
    m->st = a.take<DevState>(1);
    m->d_layers = a.take<LayerW>(L);
    if (m->fu_ok) {  // K-block-major attn_output / ffn_down, the sums and the exchange words
      m->h_fl.assign(L, FuLayer{});
      for (size_t l = 0; l < L; ++l) {
        const Q4Dev& wo = m->wo[l];
        const Q4Dev& dn = m->down[l];
        // the tensor-core copies have the same layout when their rows need no padding
        const bool share_wo = wo.qsT && wo.ldT == wo.N, share_dn = dn.qsT && dn.ldT == dn.N;
        m->h_fl[l].wo_qs = share_wo ? wo.qsT : a.take<uint4>(size_t(wo.N) * wo.nb);
        m->h_fl[l].wo_sm = share_wo ? wo.smT : a.take<uint32_t>(size_t(wo.N) * wo.nb);
        m->h_fl[l].dn_qs = share_dn ? dn.qsT : a.take<uint4>(size_t(dn.N) * dn.nb);
        m->h_fl[l].dn_sm = share_dn ? dn.smT : a.take<uint32_t>(size_t(dn.N) * dn.nb);
      }
      m->d_fl = a.take<FuLayer>(L);
      m->fya = a.take<float>(4 * d);
      m->fyb = m->fya ? m->fya + 2 * d : nullptr;
      m->fwords_n = 2 * size_t(m->sms) + 2 * size_t(m->nkv) * m->hd + size_t(m->nh) * m->fplan.S * 2 + 1;
      m->fwords = a.take<uint2>(m->fwords_n);
      m->lm_q8 = I.lm_head_bit_depth == 8 ? a.take<unsigned char>(size_t(m->Vl) * m->lm_row_bytes) : nullptr;
    }
    // LL exchange words of the persistent kernel, one contiguous range
    const size_t qd = size_t(m->nh) * m->hd, kvd = size_t(m->nkv) * m->hd;
    // the persistent kernel's split cap (plan_mega sets the same value)
    const size_t apart = size_t(m->nh) * mk_split_cap(m->nkv, m->sms) * (m->hd + 2);
    m->ll_words = 2 * d + qd + 2 * kvd + apart + size_t(m->ff) + 1 + size_t(kFlCount) * m->sms;
    uint2* llb = a.take<uint2>(m->ll_words);
    m->ll.xa = llb;
    m->ll.xb = llb + d;
    m->ll.q = llb + 2 * d;
    m->ll.kv = m->ll.q + qd;
    m->ll.apart = m->ll.kv + 2 * kvd;
    m->ll.act = m->ll.apart + apart;
    m->ll.tok = m->ll.act + m->ff;
    m->ll.flags = m->ll.tok + 1;
    if (m->max_streams > 0) {
      const size_t S = size_t(m->max_streams), G = size_t(m->nh / m->nkv);
      const size_t R = std::max(S, size_t(m->pf_rows));  // rows of a batched step or a prefill chunk
      const size_t bc = S * L * size_t(m->nkv) * m->max_ctx * m->hd;
      m->bcache.k = a.take<float>(bc);
      m->bcache.v = a.take<float>(bc);
      m->bx = a.take<float>(R * d);
      m->bq = a.take<float>(R * qd);
      m->battn = a.take<float>(R * qd);
      m->bact = a.take<float>(R * m->ff);
      m->pf_tab = a.take<unsigned>(3 * std::max<size_t>(m->pf_rows, 1));
      const size_t NS = size_t(m->nranks) * S;  // rows the lm_head of a sharded step sees
      m->blogits = a.take<float>(std::max(S * V, NS * size_t(m->Vl)));
      if (m->nranks > 1) {
        m->bxg = a.take<float>(NS * d);
        m->bkey = a.take<unsigned long long>(NS);
        m->bkey_all = a.take<unsigned long long>(NS * size_t(m->nranks));
      }
      m->bpart_o = a.take<float>(S * m->nkv * kAttnMaxSplits * G * m->hd);
      m->bpart_ml = a.take<float>(S * m->nkv * kAttnMaxSplits * G * 2);
      m->bcnt = a.take<unsigned>(S * m->nkv);
      m->blm_part = a.take<unsigned long long>(size_t(m->sms) * 4 * 16);
      m->blm_cnt = a.take<unsigned>(1);
      m->bdev = a.take<unsigned>(4 * S);
      // Q4 GEMM split partials [split][stream][row] and per-tile counters
      size_t part = 0, tiles = 0;
      const size_t shapes[4][2] = {{size_t(m->nh + 2 * m->nkv) * m->hd, size_t(d)},
                                   {size_t(d), size_t(m->nh) * m->hd},
                                   {size_t(2 * m->ff), size_t(d)},
                                   {size_t(d), size_t(m->ff)}};
      for (const auto& nk : shapes) {
        const size_t ns = (nk[1] + kSkChunk - 1) / kSkChunk;
        if (ns > 1) part = std::max(part, ns * nk[0] * R);
        tiles = std::max(tiles, (nk[0] + 2 * kSkWarps - 1) / (2 * kSkWarps) * ((R + kBatchMT - 1) / kBatchMT));
      }
      m->bsk_part = a.take<float>(std::max<size_t>(part, 1));
      m->bsk_cnt = a.take<unsigned>(tiles);
      m->bsk_tiles = tiles;
      const size_t RT = std::max(R, NS);
      if (RT >= size_t(kBatchTcMin)) {
        const size_t kmax = std::max({size_t(d), size_t(m->nh) * m->hd, size_t(m->ff)});
        m->btc_mpad = int((RT + 255) / 256 * 256);
        m->btc_hi = a.take<unsigned char>(tc_plane_bytes(m->btc_mpad, int(kmax)));
        m->btc_lo = a.take<unsigned char>(tc_plane_bytes(m->btc_mpad, int(kmax)));
        m->btc_part = a.take<float>(size_t(m->sms) * 256 * kTcRows);  // z * M * N <= SMs * NT * 128
      }
    }
  };
  {
    Arena shapes;  // a first pass fills the matrix shapes the fused plan needs
    plan(shapes);
    m->fu_ok = m->nranks == 1 && !m->has_lut && (!opts || opts->use_megakernel == 1) && plan_fused(m);
  }
  Arena sizing;
  plan(sizing);
  const size_t staging_words = (staging_bytes + 3) / 4;
  const size_t total = align_up(sizing.used, 256) + staging_words * 4 + 256;
  CK(cudaMalloc(&m->arena.base, total));
  m->arena.size = total;
  plan(m->arena);
  uint32_t* staging = m->arena.take<uint32_t>(staging_words);
  // ---- launch plans
  m->pq = plan_gemv(G_QKV, m->qkv[0], m->qkv[0].N / 2, m->sms);
  m->po = plan_gemv(G_OPROJ, m->wo[0], m->wo[0].N, m->sms);
  m->pg = plan_gemv(G_GATEUP, m->gate_up[0], m->gate_up[0].N / 2, m->sms);
  m->pd = plan_gemv(G_DOWN, m->down[0], m->down[0].N, m->sms);
  m->attn_smem = attn_smem_bytes(m->nh / m->nkv, m->hd, attn_chunk_max(m->max_ctx));
  m->lm_grid = m->sms;
  m->lm_rows = (m->V + m->lm_grid - 1) / m->lm_grid;
  m->lm_stage_n = lm_stages(m->d);
  m->lm_smem = lm_smem_bytes(m->d, m->lm_stage_n);
  if (m->lm_stage_n < 2) return set_error(GAJE_ERR_UNSUPPORTED, "n_embd too large for the lm_head ring");
  if (int s = smem_optin((const void*)k_gemv<G_QKV>, m->pq.smem)) return s;
  if (int s = smem_optin((const void*)k_gemv<G_OPROJ>, m->po.smem)) return s;
  if (int s = smem_optin((const void*)k_gemv<G_GATEUP>, m->pg.smem)) return s;
  if (int s = smem_optin((const void*)k_gemv<G_DOWN>, m->pd.smem)) return s;
  if (int s = smem_optin((const void*)k_attn, m->attn_smem)) return s;
  if (int s = smem_optin((const void*)k_lmhead, m->lm_smem)) return s;
  m->use_mega = m->nranks == 1 && !m->has_lut && (!opts || opts->use_megakernel) && plan_mega(m);
  if (m->fu_ok) {
    if (int s = smem_optin((const void*)fused_kernel(m->hd, false), m->fused_smem)) return s;
    if (int s = smem_optin((const void*)fused_kernel(m->hd, true), m->fused_smem)) return s;
    int per_sm = 0, per_sm_t = 0, coop = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fused_kernel(m->hd, false), kFuThreads, m->fused_smem));
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_t, fused_kernel(m->hd, true), kFuThreads, m->fused_smem));
    per_sm = std::min(per_sm, per_sm_t);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->device);
    m->use_fused = per_sm >= 1 && coop;
    CK(cudaMemsetAsync(m->fwords, 0, m->fwords_n * sizeof(uint2), m->stream));
  }
  if (m->use_mega) {
    if (int s = smem_optin((const void*)k_decode_mega, m->mega_smem)) return s;
    int per_sm = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_mega, kMkThreads, m->mega_smem));
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->device);
    if (per_sm < 1 || !coop) m->use_mega = false;
  }
  // zero the counters, scratch, state and caches
  CK(cudaMemsetAsync(m->attn_cnt, 0, m->nkv * sizeof(unsigned), m->stream));
  CK(cudaMemsetAsync(m->ll.xa, 0, m->ll_words * sizeof(uint2), m->stream));
  CK(cudaMemsetAsync(m->amax_cnt, 0, sizeof(unsigned), m->stream));
  if (m->max_streams > 0) {
    m->bcache.L = m->L;
    m->bcache.nkv = m->nkv;
    m->bcache.max_ctx = m->max_ctx;
    m->bcache.hd = m->hd;
    CK(cudaMemsetAsync(m->bcnt, 0, size_t(m->max_streams) * m->nkv * sizeof(unsigned), m->stream));
    CK(cudaMemsetAsync(m->blm_cnt, 0, sizeof(unsigned), m->stream));
    CK(cudaMemsetAsync(m->bsk_cnt, 0, m->bsk_tiles * sizeof(unsigned), m->stream));
    CK(cudaHostAlloc(&m->h_bdev, size_t(4) * m->max_streams * sizeof(unsigned), cudaHostAllocDefault));
    m->bpos.assign(size_t(m->max_streams), 0u);
    m->bgraphs.assign(size_t(m->max_streams) + 1, nullptr);
    if (m->pf_rows > 0)
      CK(cudaHostAlloc(&m->h_pf_tab, size_t(3) * m->pf_rows * sizeof(unsigned), cudaHostAllocDefault));
    for (cudaEvent_t& e : m->tev) CK(cudaEventCreate(&e));
    if (int s = batch_setup(m)) return s;
  }
  CK(cudaMemsetAsync(m->kcache, 0, L * size_t(m->nkv) * m->max_ctx * m->hd * 4, m->stream));
  CK(cudaMemsetAsync(m->vcache, 0, L * size_t(m->nkv) * m->max_ctx * m->hd * 4, m->stream));
  // ---- upload
  const int qkv_mode = I.rope_split ? 1 : 2;
  for (size_t l = 0; l < L; ++l) {
    const BlockRefs& b = f.blocks[l];
    if (int s = upload_matrix(m, f, b.qkv, m->qkv[l], staging, qkv_mode)) return s;
    if (int s = upload_matrix(m, f, b.wo, m->wo[l], staging, 0)) return s;
    if (int s = upload_matrix(m, f, b.gate_up, m->gate_up[l], staging, 3)) return s;
    if (int s = upload_matrix(m, f, b.down, m->down[l], staging, 0)) return s;
    CK(cudaMemcpy(m->attn_norm[l], f.blob(b.attn_norm->dna_off, d * 4), d * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(m->ffn_norm[l], f.blob(b.ffn_norm->dna_off, d * 4), d * 4, cudaMemcpyHostToDevice));
  }
  CK(cudaMemcpy(m->out_norm, f.blob(f.output_norm->dna_off, d * 4), d * 4, cudaMemcpyHostToDevice));
  // f32 rows as stored; Q8_0 rows (--quant-embed exports) dequantised to the
  // f32 values the reference computes, q * scale (blocks.rs:44-48, exact)
  auto upload_rows = [&](const FlatEntry* e, size_t r0, size_t nr, float* dst) -> int {
    if (e->bit_depth == 32) {
      CK(cudaMemcpy(dst, f.blob(e->dna_off + r0 * d * 4, nr * d * 4), nr * d * 4, cudaMemcpyHostToDevice));
      return GAJE_OK;
    }
    const size_t nb = d / 32;
    const uint8_t* src = f.blob(e->dna_off + r0 * nb * 34, nr * nb * 34);
    if (!src) return set_error(GAJE_ERR_IO, "Q8_0 rows out of range");
    std::vector<float> host(nr * d);
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)nr; ++r)
      for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = src + (size_t(r) * nb + b) * 34;
        uint16_t hs;
        memcpy(&hs, blk, 2);
        const float sc = f16_to_f32(hs);
        for (int k = 0; k < 32; ++k) host[size_t(r) * d + b * 32 + k] = float(int8_t(blk[2 + k])) * sc;
      }
    CK(cudaMemcpy(dst, host.data(), nr * d * 4, cudaMemcpyHostToDevice));
    return GAJE_OK;
  };
  if (int s = upload_rows(f.token_embd, 0, V, m->embd)) return s;
  if (int s = upload_rows(f.lm_head, size_t(m->v0), size_t(m->Vl), m->lm_head)) return s;  // this rank's rows
  if (m->lm_q8) {  // the fused kernel's Q8_0 rows: int8 codes of the row, then its f16 scales
    const size_t nb = d / 32, rb = size_t(m->lm_row_bytes), nr = size_t(m->Vl);
    const uint8_t* src = f.blob(f.lm_head->dna_off + size_t(m->v0) * nb * 34, nr * nb * 34);
    if (!src) return set_error(GAJE_ERR_IO, "Q8_0 rows out of range");
    std::vector<uint8_t> host(nr * rb, 0);
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)nr; ++r)
      for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = src + (size_t(r) * nb + b) * 34;
        uint8_t* row = host.data() + size_t(r) * rb;
        memcpy(row + b * 32, blk + 2, 32);
        memcpy(row + d + 2 * b, blk, 2);
      }
    CK(cudaMemcpy(m->lm_q8, host.data(), host.size(), cudaMemcpyHostToDevice));
  }
  if (m->lm_bias) {
    std::vector<float> b(V, 0.0f);
    memcpy(b.data(), f.blob(f.lm_head->bias_off, f.lm_head->bias_len), f.lm_head->bias_len);
    CK(cudaMemcpy(m->lm_bias, b.data() + m->v0, size_t(m->Vl) * 4, cudaMemcpyHostToDevice));
  }
  {
    std::vector<float2> rt = rope_table(m->max_ctx, m->hd, I.rope_base);
    CK(cudaMemcpy(m->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice));
  }
  {
    std::vector<LayerW> lw(L);
    for (size_t l = 0; l < L; ++l) lw[l] = m->layer(int(l));
    CK(cudaMemcpy(m->d_layers, lw.data(), L * sizeof(LayerW), cudaMemcpyHostToDevice));
  }
  for (size_t l = 0; l < L; ++l) {  // K-block-major copies for the tensor-core GEMMs' weight streams
    for (Q4Dev* q : {&m->qkv[l], &m->wo[l], &m->gate_up[l], &m->down[l]})
      if (q->qsT) k_q4_kbmajor<<<m->sms * 4, 256, 0, m->stream>>>(q->view(), q->qsT, q->smT, q->ldT);
  }
  CK(cudaGetLastError());
  if (m->fu_ok) {  // K-block-major copies of attn_output and ffn_down (shared with the above when made)
    for (size_t l = 0; l < L; ++l) {
      if (!m->wo[l].qsT)
        k_q4_kbmajor<<<m->sms * 4, 256, 0, m->stream>>>(m->wo[l].view(), const_cast<uint4*>(m->h_fl[l].wo_qs),
                                                        const_cast<uint32_t*>(m->h_fl[l].wo_sm), m->wo[l].N);
      if (!m->down[l].qsT)
        k_q4_kbmajor<<<m->sms * 4, 256, 0, m->stream>>>(m->down[l].view(), const_cast<uint4*>(m->h_fl[l].dn_qs),
                                                        const_cast<uint32_t*>(m->h_fl[l].dn_sm), m->down[l].N);
    }
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(m->d_fl, m->h_fl.data(), L * sizeof(FuLayer), cudaMemcpyHostToDevice, m->stream));
    CK(cudaStreamSynchronize(m->stream));
  }
  CK(cudaHostAlloc(&m->h_st, sizeof(DevState), cudaHostAllocDefault));
  CK(cudaHostAlloc(&m->h_tok, 64 * sizeof(unsigned), cudaHostAllocDefault));
  memset(m->h_st, 0, sizeof(DevState));
  m->h_st->nan_code = 0xFFFFFFFFu;
  CK(cudaMemcpyAsync(m->st, m->h_st, sizeof(DevState), cudaMemcpyHostToDevice, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  // ---- step parameters
  StepParams& P = m->P;
  P.d = m->d;
  P.nh = m->nh;
  P.nkv = m->nkv;
  P.hd = m->hd;
  P.ff = m->ff;
  P.V = m->V;
  P.max_ctx = m->max_ctx;
  P.n_layers = m->L;
  P.eps = I.eps;
  P.attn_scale = 1.0f / sqrtf(float(m->hd));
  P.rope_split = I.rope_split;
  P.use_genomic_norm = I.use_genomic_norm;
  P.embd = m->embd;
  P.lm_head = m->lm_head;
  P.lm_bias = m->lm_bias;
  P.lm_flush = I.lm_head_bit_depth == 8 ? 1 : 0;
  P.lm_q8 = m->lm_q8;
  P.lm_row_bytes = m->lm_q8 ? m->lm_row_bytes : int(d) * 4;
  P.out_norm = m->out_norm;
  P.rope = m->rope;
  P.x = m->x;
  P.q = m->q;
  P.attn = m->attn;
  P.act = m->act;
  P.logits = m->logits;
  P.part_o = m->part_o;
  P.part_ml = m->part_ml;
  P.attn_cnt = m->attn_cnt;
  P.amax_part = m->amax_part;
  P.amax_cnt = m->amax_cnt;
  P.tok_hist = m->tok_hist;
  P.hist_cap = unsigned(m->max_ctx);
  P.st = m->st;
  return GAJE_OK;
}

}  // namespace

extern "C" {

void gaje_load_opts_init(gaje_load_opts* o) {
  if (!o) return;
  o->device = 0;
  o->max_ctx = 4096;
  o->seed = 0;
  o->use_graph = 1;
  o->use_megakernel = 1;
  o->max_streams = 0;
  o->max_prefill = 0;
}

static int sharded_only() {
  return set_error(GAJE_ERR_UNSUPPORTED,
                   "a vocab-sharded model serves batched streams only (gaje_cuda_forward_batch / gaje_cuda_prefill)");
}

gaje_model* gaje_cuda_load(const char* flat_path, const gaje_load_opts* opts) {
  std::unique_ptr<gaje_model> m(new gaje_model());
  m->device = opts ? opts->device : 0;
  if (int s = load_impl(m.get(), flat_path, opts)) {
    (void)s;
    return nullptr;
  }
  clear_error();
  return m.release();
}

int gaje_cuda_nccl_unique_id(uint8_t* id_out) {
  if (!id_out) return set_error(GAJE_ERR_INVALID, "NULL argument");
  const NcclApi& api = nccl_api();
  if (!api.why.empty()) return set_error(GAJE_ERR_UNSUPPORTED, api.why);
  ncclUniqueId id;
  const ncclResult_t r = api.get_unique_id(&id);
  if (r != ncclSuccess) return set_error(GAJE_ERR_CUDA, std::string("ncclGetUniqueId: ") + api.error_string(r));
  static_assert(sizeof(ncclUniqueId) == GAJE_NCCL_ID_BYTES, "NCCL unique id size");
  memcpy(id_out, &id, sizeof(id));
  return GAJE_OK;
}

gaje_model* gaje_cuda_load_sharded(const char* flat_path, const gaje_load_opts* opts, int nranks, int rank,
                                   const uint8_t* nccl_id) {
  if (!nccl_id || nranks < 1 || rank < 0 || rank >= nranks) {
    set_error(GAJE_ERR_INVALID, "nranks/rank out of range or NULL nccl_id");
    return nullptr;
  }
  const NcclApi& api = nccl_api();
  if (!api.why.empty()) {
    set_error(GAJE_ERR_UNSUPPORTED, api.why);
    return nullptr;
  }
  std::unique_ptr<gaje_model> m(new gaje_model());
  m->device = opts ? opts->device : 0;
  m->nranks = nranks;
  m->rank = rank;
  if (int s = load_impl(m.get(), flat_path, opts)) {
    (void)s;
    return nullptr;
  }
  if (cudaSetDevice(m->device) != cudaSuccess) {
    set_error(GAJE_ERR_CUDA, "cudaSetDevice");
    return nullptr;
  }
  ncclUniqueId id;
  memcpy(&id, nccl_id, sizeof(id));
  const ncclResult_t r = api.comm_init_rank(&m->nccl, nranks, id, rank);
  if (r != ncclSuccess) {
    m->nccl = nullptr;
    set_error(GAJE_ERR_CUDA, std::string("ncclCommInitRank: ") + api.error_string(r));
    return nullptr;
  }
  clear_error();
  return m.release();
}

int gaje_vocab_shard(uint32_t vocab_size, int nranks, int rank, uint32_t* row0, uint32_t* rows) {
  if (!row0 || !rows || nranks < 1 || rank < 0 || rank >= nranks) return set_error(GAJE_ERR_INVALID, "bad argument");
  int r0 = 0, n = 0;
  vocab_shard(int(vocab_size), nranks, rank, r0, n);
  *row0 = uint32_t(r0);
  *rows = uint32_t(n);
  return GAJE_OK;
}

uint64_t gaje_argmax_key(float value, uint32_t index) { return host_amax_key(value, index); }
uint32_t gaje_argmax_key_index(uint64_t key) { return amax_index(key); }

void gaje_cuda_free(gaje_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  delete m;
}

int gaje_cuda_model_info(gaje_model* m, gaje_model_info* o) {
  if (!m || !o) return set_error(GAJE_ERR_INVALID, "NULL argument");
  o->vocab_size = uint32_t(m->V);
  o->n_embd = uint32_t(m->d);
  o->n_head = uint32_t(m->nh);
  o->n_head_kv = uint32_t(m->nkv);
  o->n_blocks = uint32_t(m->L);
  o->head_dim = uint32_t(m->hd);
  o->ffn_dim = uint32_t(m->ff);
  o->max_ctx = uint32_t(m->max_ctx);
  o->cache_len = m->host_pos;
  o->eps = m->info.eps;
  o->rope_base = m->info.rope_base;
  o->k_wta_ratio = m->k_wta_ratio;
  o->device_bytes = m->arena.size;
  o->grid = uint32_t(m->sms);
  o->megakernel = m->use_fused ? 2u : m->use_mega ? 1u : 0u;
  o->nranks = uint32_t(m->nranks);
  o->rank = uint32_t(m->rank);
  o->vocab_row0 = uint32_t(m->v0);
  o->vocab_rows = uint32_t(m->Vl);
  return GAJE_OK;
}

void* gaje_cuda_stream(gaje_model* m) { return m ? (void*)m->stream : nullptr; }

int gaje_cuda_clear_cache(gaje_model* m) {
  if (!m) return set_error(GAJE_ERR_INVALID, "model is NULL");
  CK(cudaSetDevice(m->device));
  if (int s = m->set_pos(0)) return s;
  CK(cudaStreamSynchronize(m->stream));
  return GAJE_OK;
}

int gaje_cuda_set_k_wta_ratio(gaje_model* m, float ratio) {
  if (!m) return set_error(GAJE_ERR_INVALID, "model is NULL");
  m->k_wta_ratio = ratio;
  m->block_k_wta_ratio = ratio;
  return GAJE_OK;
}

int gaje_cuda_set_seed(gaje_model* m, uint64_t seed) {
  if (!m) return set_error(GAJE_ERR_INVALID, "model is NULL");
  m->rng.s = seed;
  return GAJE_OK;
}

int gaje_cuda_forward(gaje_model* m, uint32_t token_id, int clear_cache, float* logits_out,
                      uint32_t* argmax_out) {
  if (!m) return set_error(GAJE_ERR_INVALID, "model is NULL");
  if (m->nranks > 1) return sharded_only();
  CK(cudaSetDevice(m->device));
  if (clear_cache)
    if (int s = m->set_pos(0)) return s;
  if (m->host_pos >= uint32_t(m->max_ctx))
    return set_error(GAJE_ERR_CONTEXT, "KV cache is full (max_ctx positions)");
  m->h_tok[0] = token_id;
  CK(cudaMemcpyAsync(&m->st->token, m->h_tok, 4, cudaMemcpyHostToDevice, m->stream));
  if (int s = m->run_steps(1)) return s;
  CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, m->stream));
  if (logits_out) CK(cudaMemcpyAsync(logits_out, m->logits, size_t(m->V) * 4, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  m->host_pos += 1;
  if (int s = m->check_state()) return s;
  if (argmax_out) *argmax_out = m->h_st->argmax;
  return GAJE_OK;
}

int gaje_cuda_forward_batch(gaje_model* m, const uint32_t* stream_ids, const uint32_t* tokens, size_t B,
                            uint32_t* argmax_out, float* logits_out) {
  if (!m || (B && (!stream_ids || !tokens))) return set_error(GAJE_ERR_INVALID, "NULL argument");
  if (B == 0) return GAJE_OK;
  if (m->max_streams <= 0)
    return set_error(GAJE_ERR_INVALID, "the model was loaded without batched streams (gaje_load_opts.max_streams)");
  if (B > size_t(m->max_streams)) return set_error(GAJE_ERR_INVALID, "more streams in the batch than max_streams");
  if (m->block_k() > 0)
    return set_error(GAJE_ERR_UNSUPPORTED, "block K-WTA is not implemented on the batched path");
  if (m->info.use_genomic_norm)
    return set_error(GAJE_ERR_UNSUPPORTED, "use_genomic_norm is not implemented on the batched path");
  if (m->nranks > 1) {
    if (logits_out)
      return set_error(GAJE_ERR_UNSUPPORTED, "a vocab-sharded model returns argmax only (no full-vocabulary logits)");
    if (!m->nccl) return set_error(GAJE_ERR_CUDA, "the sharded group failed earlier; reload the model");
  }
  const size_t S = size_t(m->max_streams);
  std::vector<char> seen(S, 0);
  for (size_t b = 0; b < B; ++b) {
    const uint32_t sid = stream_ids[b];
    if (sid >= S) return set_error(GAJE_ERR_INVALID, "stream id out of range");
    if (seen[sid]) return set_error(GAJE_ERR_INVALID, "a stream appears twice in one batch");
    seen[sid] = 1;
    if (m->bpos[sid] >= uint32_t(m->max_ctx)) return set_error(GAJE_ERR_CONTEXT, "KV cache full (max_ctx positions)");
    m->h_bdev[b] = tokens[b];
    m->h_bdev[S + b] = m->bpos[sid];
    m->h_bdev[2 * S + b] = sid;
  }
  CK(cudaSetDevice(m->device));
  cudaStream_t st = m->stream;
  const int Bi = int(B);
  CK(cudaMemcpyAsync(m->bdev, m->h_bdev, 3 * S * sizeof(unsigned), cudaMemcpyHostToDevice, st));
  const bool timed = m->tev[0] != nullptr;
  if (timed) CK(cudaEventRecord(m->tev[0], st));
  if (!m->use_graph) {
    if (int s = launch_batch(m, Bi)) return s;
  } else {
    cudaGraphExec_t& ge = m->bgraphs[size_t(Bi)];
    if (!ge) {
      cudaGraph_t g = nullptr;
      CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      const int s = launch_batch(m, Bi);
      const cudaError_t e = cudaStreamEndCapture(st, &g);
      if (s) {
        if (g) cudaGraphDestroy(g);
        return s;
      }
      if (e != cudaSuccess) return set_error(GAJE_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
      const cudaError_t ei = cudaGraphInstantiate(&ge, g, 0);
      cudaGraphDestroy(g);
      if (ei != cudaSuccess) {
        ge = nullptr;
        return set_error(GAJE_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ei));
      }
    }
    CK(cudaGraphLaunch(ge, st));
  }
  if (timed) CK(cudaEventRecord(m->tev[1], st));
  if (m->nranks > 1) {  // the collective head: every rank's rows through this rank's vocab rows
    if (int s = sharded_head(m, m->bx, Bi, m->bdev + 3 * S)) return s;
  } else if (timed) {  // one GPU: the head ran inside the step graph
    for (int k = 2; k < 5; ++k) CK(cudaEventRecord(m->tev[k], st));
  }
  const int kk = m->logits_k();
  if (logits_out && kk > 0)  // K-WTA on the returned logits (llm/forward.rs:58-61); the argmax is unaffected
    for (int b = 0; b < Bi; ++b) k_kwta<<<1, kKwtaThreads, 0, st>>>(m->blogits + size_t(b) * m->V, m->V, kk);
  CK(cudaMemcpyAsync(m->h_bdev + 3 * S, m->bdev + 3 * S, B * sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  if (logits_out)
    CK(cudaMemcpyAsync(logits_out, m->blogits, B * size_t(m->V) * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, st));
  if (m->nranks > 1) {
    if (int s = sync_sharded(m)) return s;
  } else {
    CK(cudaStreamSynchronize(st));
  }
  if (timed) {
    for (int k = 0; k < 4; ++k) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, m->tev[k], m->tev[k + 1]) == cudaSuccess) m->tacc[k] += ms;
    }
    m->tcount += 1;
  }
  for (size_t b = 0; b < B; ++b) m->bpos[stream_ids[b]] += 1u;
  if (argmax_out)
    for (size_t b = 0; b < B; ++b) argmax_out[b] = m->h_bdev[3 * S + b];
  return m->check_state();
}

int gaje_cuda_batch_timings(gaje_model* m, float* ms_out, uint32_t* steps_out, int reset) {
  if (!m || !ms_out) return set_error(GAJE_ERR_INVALID, "NULL argument");
  if (!m->tev[0]) return set_error(GAJE_ERR_INVALID, "the model was loaded without batched streams");
  for (int k = 0; k < 4; ++k) ms_out[k] = float(m->tacc[k]);
  if (steps_out) *steps_out = m->tcount;
  if (reset) {
    for (double& v : m->tacc) v = 0.0;
    m->tcount = 0;
  }
  return GAJE_OK;
}

int gaje_cuda_profile_batch(gaje_model* m, const uint32_t* stream_ids, const uint32_t* tokens, size_t B, float* ms,
                            uint32_t* launches) {
  if (!m || !B || !stream_ids || !tokens) return set_error(GAJE_ERR_INVALID, "NULL argument");
  if (m->max_streams <= 0 || B > size_t(m->max_streams)) return set_error(GAJE_ERR_INVALID, "bad batch size");
  if (m->nranks > 1) return set_error(GAJE_ERR_UNSUPPORTED, "profile a single-GPU model");
  if (m->block_k() > 0 || m->info.use_genomic_norm)
    return set_error(GAJE_ERR_UNSUPPORTED, "block K-WTA / use_genomic_norm are not implemented on the batched path");
  const size_t S = size_t(m->max_streams);
  std::vector<char> seen(S, 0);
  for (size_t b = 0; b < B; ++b) {
    const uint32_t sid = stream_ids[b];
    if (sid >= S || seen[sid]) return set_error(GAJE_ERR_INVALID, "stream ids must be distinct and < max_streams");
    seen[sid] = 1;
    if (m->bpos[sid] >= uint32_t(m->max_ctx)) return set_error(GAJE_ERR_CONTEXT, "KV cache full (max_ctx positions)");
    m->h_bdev[b] = tokens[b];
    m->h_bdev[S + b] = m->bpos[sid];
    m->h_bdev[2 * S + b] = sid;
  }
  CK(cudaSetDevice(m->device));
  CK(cudaMemcpyAsync(m->bdev, m->h_bdev, 3 * S * sizeof(unsigned), cudaMemcpyHostToDevice, m->stream));
  StepProf prof;
  CK(cudaEventCreate(&prof.e0));
  CK(cudaEventCreate(&prof.e1));
  const int s = launch_batch(m, int(B), &prof);
  cudaEventDestroy(prof.e0);
  cudaEventDestroy(prof.e1);
  if (s) return s;
  CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  for (size_t b = 0; b < B; ++b) m->bpos[stream_ids[b]] += 1u;
  for (int k = 0; k < GAJE_K_COUNT; ++k) {
    if (ms) ms[k] = prof.ms[k];
    if (launches) launches[k] = prof.n[k];
  }
  return m->check_state();
}

int gaje_cuda_prefill(gaje_model* m, uint32_t stream_id, const uint32_t* tokens, size_t n, uint32_t* argmax_out,
                      float* logits_out) {
  if (!m || (n && !tokens)) return set_error(GAJE_ERR_INVALID, "NULL argument");
  if (n == 0) return GAJE_OK;
  if (m->pf_rows <= 0)
    return set_error(GAJE_ERR_INVALID, "the model was loaded without prefill rows (gaje_load_opts.max_prefill)");
  if (stream_id >= uint32_t(m->max_streams)) return set_error(GAJE_ERR_INVALID, "stream id out of range");
  if (m->block_k() > 0)
    return set_error(GAJE_ERR_UNSUPPORTED, "block K-WTA is not implemented on the batched path");
  if (m->info.use_genomic_norm)
    return set_error(GAJE_ERR_UNSUPPORTED, "use_genomic_norm is not implemented on the batched path");
  if (size_t(m->bpos[stream_id]) + n > size_t(m->max_ctx))
    return set_error(GAJE_ERR_CONTEXT, "KV cache would overflow (max_ctx positions)");
  if (m->nranks > 1) {
    if (logits_out)
      return set_error(GAJE_ERR_UNSUPPORTED, "a vocab-sharded model returns argmax only (no full-vocabulary logits)");
    if (!m->nccl) return set_error(GAJE_ERR_CUDA, "the sharded group failed earlier; reload the model");
  }
  CK(cudaSetDevice(m->device));
  cudaStream_t st = m->stream;
  const size_t R = size_t(m->pf_rows);
  int last_nc = 0;
  for (size_t c0 = 0; c0 < n; c0 += R) {
    const int nc = int(std::min(R, n - c0));
    const unsigned p0 = m->bpos[stream_id];
    if (c0 > 0) CK(cudaStreamSynchronize(st));  // the pinned table is reused by the next chunk
    for (int i = 0; i < nc; ++i) {
      m->h_pf_tab[i] = tokens[c0 + size_t(i)];
      m->h_pf_tab[R + size_t(i)] = p0 + unsigned(i);
      m->h_pf_tab[2 * R + size_t(i)] = stream_id;
    }
    CK(cudaMemcpyAsync(m->pf_tab, m->h_pf_tab, 3 * R * sizeof(unsigned), cudaMemcpyHostToDevice, st));
    if (int s = launch_prefill_chunk(m, nc, int(p0), stream_id, c0 + size_t(nc) == n)) return s;
    m->bpos[stream_id] += unsigned(nc);
    last_nc = nc;
  }
  const size_t S = size_t(m->max_streams);
  if (m->nranks > 1)  // the collective head on the prompt's last row
    if (int s = sharded_head(m, m->bx + size_t(last_nc - 1) * m->d, 1, m->bdev + 3 * S)) return s;
  const int kk = m->logits_k();
  if (logits_out && kk > 0) k_kwta<<<1, kKwtaThreads, 0, st>>>(m->blogits, m->V, kk);
  CK(cudaMemcpyAsync(m->h_bdev + 3 * S, m->bdev + 3 * S, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  if (logits_out) CK(cudaMemcpyAsync(logits_out, m->blogits, size_t(m->V) * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, st));
  if (m->nranks > 1) {
    if (int s = sync_sharded(m)) return s;
  } else {
    CK(cudaStreamSynchronize(st));
  }
  if (argmax_out) *argmax_out = m->h_bdev[3 * S];
  return m->check_state();
}

int gaje_cuda_clear_stream(gaje_model* m, uint32_t stream_id) {
  if (!m) return set_error(GAJE_ERR_INVALID, "model is NULL");
  if (stream_id >= uint32_t(std::max(0, m->max_streams))) return set_error(GAJE_ERR_INVALID, "stream id out of range");
  m->bpos[stream_id] = 0;
  return GAJE_OK;
}

int gaje_cuda_stream_len(gaje_model* m, uint32_t stream_id, uint32_t* len) {
  if (!m || !len) return set_error(GAJE_ERR_INVALID, "NULL argument");
  if (stream_id >= uint32_t(std::max(0, m->max_streams))) return set_error(GAJE_ERR_INVALID, "stream id out of range");
  *len = m->bpos[stream_id];
  return GAJE_OK;
}

int gaje_cuda_decode_greedy(gaje_model* m, uint32_t first_token, size_t n_steps, uint32_t* tokens_out) {
  if (!m) return set_error(GAJE_ERR_INVALID, "model is NULL");
  if (m->nranks > 1) return sharded_only();
  CK(cudaSetDevice(m->device));
  if (size_t(m->host_pos) + n_steps > size_t(m->max_ctx))
    return set_error(GAJE_ERR_CONTEXT, "KV cache would overflow (max_ctx positions)");
  m->h_st->token = first_token;
  m->h_st->hist_len = 0;
  CK(cudaMemcpyAsync(&m->st->token, &m->h_st->token, 4, cudaMemcpyHostToDevice, m->stream));
  CK(cudaMemcpyAsync(&m->st->hist_len, &m->h_st->hist_len, 4, cudaMemcpyHostToDevice, m->stream));
  if (int s = m->run_steps(n_steps)) return s;
  CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, m->stream));
  if (tokens_out && n_steps)
    CK(cudaMemcpyAsync(tokens_out, m->tok_hist, n_steps * 4, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  m->host_pos += uint32_t(n_steps);
  return m->check_state();
}

int gaje_cuda_profile_steps(gaje_model* m, uint32_t first_token, size_t n_steps, float* ms,
                            uint32_t* launches) {
  if (!m) return set_error(GAJE_ERR_INVALID, "model is NULL");
  if (m->nranks > 1) return sharded_only();
  CK(cudaSetDevice(m->device));
  if (size_t(m->host_pos) + n_steps > size_t(m->max_ctx))
    return set_error(GAJE_ERR_CONTEXT, "KV cache would overflow (max_ctx positions)");
  float acc[GAJE_K_COUNT] = {0};
  uint32_t cnt[GAJE_K_COUNT] = {0};
  m->h_st->token = first_token;
  m->h_st->hist_len = 0;
  CK(cudaMemcpyAsync(&m->st->token, &m->h_st->token, 4, cudaMemcpyHostToDevice, m->stream));
  CK(cudaMemcpyAsync(&m->st->hist_len, &m->h_st->hist_len, 4, cudaMemcpyHostToDevice, m->stream));
  for (size_t i = 0; i < n_steps; ++i)
    if (int s = m->launch_step(m->logits_k(), m->block_k(), acc, cnt)) return s;
  CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  m->host_pos += uint32_t(n_steps);
  for (int c = 0; c < GAJE_K_COUNT; ++c) {
    if (ms) ms[c] = n_steps ? acc[c] / float(n_steps) : 0.f;
    if (launches) launches[c] = n_steps ? uint32_t(cnt[c] / n_steps) : 0u;
  }
  return m->check_state();
}

// Runs n_steps greedy steps in one launch of the persistent kernel with the
// phase stamps of CTA 0 (stamps, [n_steps][5L+1]) and, when trace is non-null,
// every CTA's in-phase stamps ([grid][n_steps][5L+1][kMkTrace]) copied to the
// host vectors.
static int mega_stamped_run(gaje_model* m, uint32_t first_token, size_t n_steps, bool want_trace,
                            std::vector<unsigned long long>& ts, std::vector<unsigned long long>* tr) {
  if (!m->use_mega) return set_error(GAJE_ERR_UNSUPPORTED, "the model runs on the kernel-per-phase engine");
  CK(cudaSetDevice(m->device));
  if (size_t(m->host_pos) + n_steps > size_t(m->max_ctx))
    return set_error(GAJE_ERR_CONTEXT, "KV cache would overflow (max_ctx positions)");
  if (want_trace && n_steps > 4096) return set_error(GAJE_ERR_INVALID, "a trace covers at most 4096 steps");
  const size_t per = size_t(5 * m->L + 1), need = n_steps * per + 1;
  if (m->phase_ns_cap < need) {
    if (m->phase_ns) cudaFree(m->phase_ns);
    m->phase_ns = nullptr;
    CK(cudaMalloc(&m->phase_ns, need * 8));
    m->phase_ns_cap = need;
  }
  const size_t tneed = want_trace ? size_t(m->sms) * n_steps * per * kMkTrace : 0;
  if (want_trace && m->trace_ns_cap < tneed) {
    if (m->trace_ns) cudaFree(m->trace_ns);
    m->trace_ns = nullptr;
    CK(cudaMalloc(&m->trace_ns, tneed * 8));
    m->trace_ns_cap = tneed;
  }
  m->h_st->token = first_token;
  m->h_st->hist_len = 0;
  CK(cudaMemcpyAsync(&m->st->token, &m->h_st->token, 4, cudaMemcpyHostToDevice, m->stream));
  CK(cudaMemcpyAsync(&m->st->hist_len, &m->h_st->hist_len, 4, cudaMemcpyHostToDevice, m->stream));
  if (want_trace) CK(cudaMemsetAsync(m->trace_ns, 0, tneed * 8, m->stream));
  if (int s = m->run_steps(n_steps, m->phase_ns, want_trace ? m->trace_ns : nullptr)) return s;
  ts.assign(n_steps * per, 0ull);
  CK(cudaMemcpyAsync(ts.data(), m->phase_ns, ts.size() * 8, cudaMemcpyDeviceToHost, m->stream));
  if (want_trace) {
    tr->assign(tneed, 0ull);
    CK(cudaMemcpyAsync(tr->data(), m->trace_ns, tneed * 8, cudaMemcpyDeviceToHost, m->stream));
  }
  CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  m->host_pos += uint32_t(n_steps);
  return m->check_state();
}

int gaje_cuda_profile_phases(gaje_model* m, uint32_t first_token, size_t n_steps, float* us, float* step_us,
                             float* detail_us) {
  if (!m) return set_error(GAJE_ERR_INVALID, "model is NULL");
  if (m->nranks > 1) return sharded_only();
  if (n_steps == 0) return GAJE_OK;
  std::vector<unsigned long long> ts, tr;
  if (int s = mega_stamped_run(m, first_token, n_steps, detail_us != nullptr, ts, &tr)) return s;
  const size_t per = size_t(5 * m->L + 1);
  // the first phase of a launch has no start stamp (a kernel to take one
  // would perturb the timing): step 0 is skipped in the means
  double acc[GAJE_PH_COUNT] = {0}, step = 0;
  size_t counted = 0;
  for (size_t s = 1; s < n_steps; ++s) {
    unsigned long long prev = ts[(s - 1) * per + per - 1];
    const unsigned long long start = prev;
    for (size_t k = 0; k < per; ++k) {
      const unsigned long long t = ts[s * per + k];
      const int ph = k + 1 == per ? GAJE_PH_LMHEAD : int(k % 5);
      acc[ph] += double(t - prev);
      prev = t;
    }
    step += double(prev - start);
    ++counted;
  }
  for (int k = 0; k < GAJE_PH_COUNT; ++k) us[k] = counted ? float(acc[k] / counted / 1000.0) : 0.f;
  if (step_us) *step_us = counted ? float(step / counted / 1000.0) : 0.f;
  if (detail_us) {
    // CTA 0, per phase kind: [previous phase done, trace points 0-4] -> 5
    // intervals; a missing point (no work of that kind) counts as zero time
    constexpr int kPts = 5;
    double dacc[GAJE_PH_COUNT * kPts] = {0};
    for (size_t st = 1; st < n_steps; ++st)
      for (size_t k = 0; k < per; ++k) {
        const int ph = k + 1 == per ? GAJE_PH_LMHEAD : int(k % 5);
        unsigned long long pts[kPts + 1];
        pts[0] = ts[st * per + k - 1];
        for (int j = 0; j < kPts; ++j) pts[1 + j] = tr[(st * per + k) * kMkTrace + j];
        for (int j = 0; j < kPts; ++j) {
          const unsigned long long a = pts[j], b = pts[j + 1];
          if (a && b && b >= a) dacc[ph * kPts + j] += double(b - a);
          else if (a && !b) pts[j + 1] = a;
        }
      }
    for (int i = 0; i < GAJE_PH_COUNT * kPts; ++i)
      detail_us[i] = counted ? float(dacc[i] / counted / 1000.0) : 0.f;
  }
  return GAJE_OK;
}

int gaje_cuda_trace_steps(gaje_model* m, uint32_t first_token, size_t n_steps, uint64_t* out, size_t out_len,
                          size_t* n_written) {
  if (!m || !n_written || (out_len && !out)) return set_error(GAJE_ERR_INVALID, "NULL argument");
  *n_written = 0;
  if (m->nranks > 1) return sharded_only();
  if (n_steps == 0) return GAJE_OK;
  const size_t need = size_t(m->sms) * n_steps * size_t(5 * m->L + 1) * kMkTrace;
  if (out_len < need) return set_error(GAJE_ERR_INVALID, "trace buffer too small: need grid*n_steps*(5L+1)*6 words");
  std::vector<unsigned long long> ts, tr;
  if (int s = mega_stamped_run(m, first_token, n_steps, true, ts, &tr)) return s;
  std::memcpy(out, tr.data(), need * 8);
  *n_written = need;
  return GAJE_OK;
}

int gaje_cuda_set_wait_limit(int device, uint64_t ns) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n)
    return set_error(GAJE_ERR_INVALID, "no such CUDA device");
  const unsigned long long v = ns ? (unsigned long long)ns : kWaitNsDefault;
  CK(cudaSetDevice(device));
  CK(cudaMemcpyToSymbol(c_wait_ns, &v, sizeof(v)));
  CK(cudaDeviceSynchronize());
  return GAJE_OK;
}

int gaje_cuda_debug_withhold_flag(gaje_model* m, int cta) {
  if (!m) return set_error(GAJE_ERR_INVALID, "NULL argument");
  if (!m->use_fused) return set_error(GAJE_ERR_UNSUPPORTED, "the model does not run the two-exchange kernel");
  if (cta < 0 || cta >= int(m->fplan.nA)) return set_error(GAJE_ERR_INVALID, "cta must be an attention CTA");
  m->withhold_cta = cta;
  return GAJE_OK;
}

int gaje_cuda_trace_fused(gaje_model* m, uint32_t first_token, size_t n_steps, uint64_t* out, size_t out_len,
                          size_t* n_written) {
  if (!m || !n_written || (out_len && !out)) return set_error(GAJE_ERR_INVALID, "NULL argument");
  *n_written = 0;
  if (!m->use_fused) return set_error(GAJE_ERR_UNSUPPORTED, "the model does not run the two-exchange kernel");
  if (n_steps == 0 || n_steps > 4096) return set_error(GAJE_ERR_INVALID, "n_steps must be in 1..4096");
  const size_t need = size_t(m->sms) * n_steps * size_t(m->L + 1) * kFuTrace;
  if (out_len < need) return set_error(GAJE_ERR_INVALID, "out_len too small");
  CK(cudaSetDevice(m->device));
  if (size_t(m->host_pos) + n_steps > size_t(m->max_ctx))
    return set_error(GAJE_ERR_CONTEXT, "KV cache would overflow (max_ctx positions)");
  if (m->trace_ns_cap < need) {
    if (m->trace_ns) cudaFree(m->trace_ns);
    m->trace_ns = nullptr;
    m->trace_ns_cap = 0;
    CK(cudaMalloc(&m->trace_ns, need * sizeof(unsigned long long)));
    m->trace_ns_cap = need;
  }
  CK(cudaMemsetAsync(m->trace_ns, 0, need * sizeof(unsigned long long), m->stream));
  m->h_st->token = first_token;
  CK(cudaMemcpyAsync(&m->st->token, &m->h_st->token, 4, cudaMemcpyHostToDevice, m->stream));
  if (int s = m->run_fused(n_steps, m->trace_ns)) return s;
  CK(cudaMemcpyAsync(out, m->trace_ns, need * sizeof(unsigned long long), cudaMemcpyDeviceToHost, m->stream));
  CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  m->host_pos += uint32_t(n_steps);
  *n_written = need;
  return m->check_state();
}

int gaje_cuda_generate(gaje_model* m, const uint32_t* prompt, size_t n_prompt, size_t max_new,
                       float temperature, float rep_penalty, const uint32_t* eos, size_t n_eos,
                       uint32_t* out, size_t* n_out) {
  if (!m || !n_out || (n_prompt && !prompt) || (n_eos && !eos) || (max_new && !out))
    return set_error(GAJE_ERR_INVALID, "NULL argument");
  if (m->nranks > 1) return sharded_only();
  *n_out = 0;
  if (n_prompt == 0) return set_error(GAJE_ERR_INVALID, "Prompt tokens cannot be empty");
  CK(cudaSetDevice(m->device));
  if (n_prompt + max_new > size_t(m->max_ctx))
    return set_error(GAJE_ERR_CONTEXT, "prompt + max_new exceeds max_ctx");
  if (int s = m->set_pos(0)) return s;
  // prefill token by token, as the reference does
  for (size_t i = 0; i < n_prompt; ++i) {
    m->h_tok[0] = prompt[i];
    CK(cudaMemcpyAsync(&m->st->token, m->h_tok, 4, cudaMemcpyHostToDevice, m->stream));
    if (int s = m->run_steps(1)) return s;
    CK(cudaStreamSynchronize(m->stream));  // h_tok is reused
    m->host_pos += 1;
  }
  CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  if (int s = m->check_state()) return s;
  std::vector<uint32_t> gen;
  std::set<uint32_t> eos_set(eos, eos + n_eos);
  std::vector<unsigned> seen_host;
  for (size_t step = 0; step < max_new; ++step) {
    uint32_t next;
    const bool penal = rep_penalty > 1.0f;
    if (penal) {
      std::set<uint32_t> seen(gen.begin(), gen.end());
      for (uint32_t e : eos_set) seen.erase(e);
      seen_host.assign(seen.begin(), seen.end());
      if (!seen_host.empty()) {
        CK(cudaMemcpyAsync(m->pen_ids, seen_host.data(), seen_host.size() * 4, cudaMemcpyHostToDevice, m->stream));
        k_penalty<<<1, 256, 0, m->stream>>>(m->logits, m->V, m->pen_ids, int(seen_host.size()), rep_penalty);
        CK(cudaGetLastError());
      }
    }
    if (temperature <= 1e-5f) {
      if (penal) {
        k_select<<<1, 1024, 0, m->stream>>>(m->logits, m->V, 0, 1.0f, 0.0f, m->sel_out);
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(m->h_tok, m->sel_out, 4, cudaMemcpyDeviceToHost, m->stream));
        CK(cudaStreamSynchronize(m->stream));
        next = m->h_tok[0];
      } else {
        next = m->h_st->argmax;  // the lm_head kernel's first-max argmax
      }
    } else {
      const float r = m->rng.uniform();
      k_select<<<1, 1024, 0, m->stream>>>(m->logits, m->V, 1, temperature, r, m->sel_out);
      CK(cudaGetLastError());
      CK(cudaMemcpyAsync(m->h_tok, m->sel_out, 4, cudaMemcpyDeviceToHost, m->stream));
      CK(cudaStreamSynchronize(m->stream));
      next = m->h_tok[0];
    }
    gen.push_back(next);
    if (eos_set.count(next)) break;
    bool repeated = false;
    for (size_t w = 2; w <= 48 && !repeated; ++w) {
      if (gen.size() >= w * 3) {
        const size_t L = gen.size();
        repeated = std::equal(gen.begin() + (L - w), gen.end(), gen.begin() + (L - 2 * w)) &&
                   std::equal(gen.begin() + (L - w), gen.end(), gen.begin() + (L - 3 * w));
      }
    }
    if (repeated) break;
    if (m->host_pos >= uint32_t(m->max_ctx)) return set_error(GAJE_ERR_CONTEXT, "KV cache is full");
    m->h_tok[0] = next;
    CK(cudaMemcpyAsync(&m->st->token, m->h_tok, 4, cudaMemcpyHostToDevice, m->stream));
    if (int s = m->run_steps(1)) return s;
    CK(cudaMemcpyAsync(m->h_st, m->st, sizeof(DevState), cudaMemcpyDeviceToHost, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    m->host_pos += 1;
    if (int s = m->check_state()) return s;
  }
  for (size_t i = 0; i < gen.size(); ++i) out[i] = gen[i];
  *n_out = gen.size();
  clear_error();
  return GAJE_OK;
}

}  // extern "C"

// ================================================================ op level
struct gaje_q4_matrix {
  int device = 0;
  Q4Dev m;
  void* mem = nullptr;
};

namespace {

// One scratch area per device for the op-level entry points, shared by every
// op call on that device: a DevState for status words, argmax partials and
// the attention split partials.  Op calls that overlap on the GPU race on it.
struct OpWorkspace {
  std::mutex mu;
  void* mem = nullptr;
  size_t size = 0;
};
OpWorkspace g_ws[64];
OpWorkspace g_ws_tc[64];  // the tensor-core GEMM op: [split-K partials][split planes]
// layout: [DevState][argmax partials, kWsArgmaxParts x u64][argmax counter]
//         then, from kWsAttnBase: [attention counters][timeout marks][part_ml][part_o]
constexpr size_t kWsArgmaxParts = 4096;
constexpr size_t kWsPartsOff = 256;
constexpr size_t kWsCntOff = kWsPartsOff + kWsArgmaxParts * 8;
constexpr size_t kWsAttnBase = kWsCntOff + 4096;

int ws_get(int dev, size_t bytes, char** out, OpWorkspace* pool = g_ws) {
  if (dev < 0 || dev >= 64) return set_error(GAJE_ERR_INVALID, "device ordinal out of range");
  OpWorkspace& w = pool[dev];
  std::lock_guard<std::mutex> lk(w.mu);
  if (w.size < bytes) {
    if (w.mem) {
      cudaDeviceSynchronize();
      cudaFree(w.mem);
      w.mem = nullptr;
      w.size = 0;
    }
    CK(cudaMalloc(&w.mem, bytes));
    CK(cudaMemset(w.mem, 0, bytes));
    w.size = bytes;
  }
  *out = static_cast<char*>(w.mem);
  return GAJE_OK;
}

int sm_count(int dev) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

extern "C" {

gaje_q4_matrix* gaje_cuda_q4_0_upload(const uint8_t* blocks, size_t N, size_t K, const float* bias, int device) {
  if (!blocks || !N || !K || K % 32 || N > 0x7FFFFFFF || K > 0x7FFFFFFF) {
    set_error(GAJE_ERR_INVALID, "blocks must be non-NULL with K a multiple of 32");
    return nullptr;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    set_error(GAJE_ERR_CUDA, "cudaSetDevice failed");
    return nullptr;
  }
  std::unique_ptr<gaje_q4_matrix> h(new gaje_q4_matrix());
  h->device = device;
  const size_t nb = K / 32, nbp = (nb + 3) / 4 * 4, nblk = N * nb;
  uint32_t* raw = nullptr;
  const size_t ldT = (N + 3) / 4 * 4;
  auto carve = [&](Arena& ar) {
    h->m.qs = ar.take<uint4>(nblk);
    h->m.sm = ar.take<uint32_t>(N * nbp);
    h->m.bias = bias ? ar.take<float>(N) : nullptr;
    h->m.qsT = ar.take<uint4>(ldT * nb);  // the tensor-core path's weight stream (M >= 16)
    h->m.smT = ar.take<uint32_t>(ldT * nb);
    raw = ar.take<uint32_t>(nblk * 5);
  };
  Arena a;
  carve(a);
  if (cudaMalloc(&h->mem, a.used) != cudaSuccess) {
    set_error(GAJE_ERR_CUDA, "cudaMalloc failed");
    return nullptr;
  }
  Arena b;
  b.base = static_cast<char*>(h->mem);
  carve(b);
  h->m.N = int(N);
  h->m.K = int(K);
  h->m.nb = int(nb);
  h->m.nbp = int(nbp);
  h->m.ldT = int(ldT);
  if (cudaMemcpy(raw, blocks, nblk * 20, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(h->m.sm, 0, N * nbp * 4) != cudaSuccess ||
      (bias && cudaMemcpy(h->m.bias, bias, N * 4, cudaMemcpyHostToDevice) != cudaSuccess)) {
    cudaFree(h->mem);
    set_error(GAJE_ERR_CUDA, "upload failed");
    return nullptr;
  }
  k_repack_q4<<<int(std::min<size_t>((nblk + 255) / 256, 8192)), 256>>>(raw, int(N), int(nb), int(nbp), 0, 0, 0,
                                                                        h->m.qs, h->m.sm);
  k_q4_kbmajor<<<int(std::min<size_t>((nblk + 255) / 256, 8192)), 256>>>(h->m.view(), h->m.qsT, h->m.smT, int(ldT));
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(h->mem);
    set_error(GAJE_ERR_CUDA, "repack failed");
    return nullptr;
  }
  clear_error();
  return h.release();
}

gaje_q4_matrix* gaje_cuda_lut4_upload(const uint8_t* nibbles, const float* centroids, size_t n_centroids, size_t N,
                                      size_t K, const float* bias, int device) {
  if (!nibbles || !centroids || !N || !K || K % 32 || N > 0x7FFFFFFF || K > 0x7FFFFFFF) {
    set_error(GAJE_ERR_INVALID, "nibbles / centroids must be non-NULL with K a multiple of 32");
    return nullptr;
  }
  const size_t nb = K / 32;
  if (n_centroids != 16 && n_centroids != nb * 16 && n_centroids != N * nb * 16) {
    set_error(GAJE_ERR_SHAPE, "unsupported centroid count (16, K/32*16 or N*K/32*16)");
    return nullptr;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    set_error(GAJE_ERR_CUDA, "cudaSetDevice failed");
    return nullptr;
  }
  std::unique_ptr<gaje_q4_matrix> h(new gaje_q4_matrix());
  h->device = device;
  auto carve = [&](Arena& ar) {
    h->m.qs = ar.take<uint4>(N * nb);
    h->m.lut = ar.take<float>(N * nb * 16);
    h->m.bias = bias ? ar.take<float>(N) : nullptr;
  };
  Arena a;
  carve(a);
  if (cudaMalloc(&h->mem, a.used) != cudaSuccess) {
    set_error(GAJE_ERR_CUDA, "cudaMalloc failed");
    return nullptr;
  }
  Arena b;
  b.base = static_cast<char*>(h->mem);
  carve(b);
  h->m.sm = nullptr;
  h->m.N = int(N);
  h->m.K = int(K);
  h->m.nb = int(nb);
  h->m.nbp = int((nb + 3) / 4 * 4);
  std::vector<uint32_t> words;
  std::vector<float> lut;
  lut4_rows_host(nibbles, centroids, n_centroids, int(N), int(K), 0, 0, words, lut);
  if (cudaMemcpy(h->m.qs, words.data(), words.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(h->m.lut, lut.data(), lut.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      (bias && cudaMemcpy(h->m.bias, bias, N * 4, cudaMemcpyHostToDevice) != cudaSuccess)) {
    cudaFree(h->mem);
    set_error(GAJE_ERR_CUDA, "upload failed");
    return nullptr;
  }
  clear_error();
  return h.release();
}

void gaje_cuda_q4_0_release(gaje_q4_matrix* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  cudaFree(h->mem);
  delete h;
}

int gaje_cuda_q4_0_gemv(const gaje_q4_matrix* h, const float* x, float* y, size_t M, void* stream) {
  if (!h || !x || !y) return set_error(GAJE_ERR_INVALID, "NULL argument");
  if (M == 0) return GAJE_OK;
  if (M > 65535) return set_error(GAJE_ERR_INVALID, "M above 65535");
  CK(cudaSetDevice(h->device));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 1 || h->m.lut) {  // the decode kernel itself (staged rows); a Genomic4Bit table: once per vector
    char* ws;
    if (int st = ws_get(h->device, kWsAttnBase, &ws)) return st;
    GemvPlan p = plan_gemv(G_PLAIN, h->m, h->m.N, sm_count(h->device));
    if (int st = smem_optin((const void*)k_gemv<G_PLAIN>, p.smem)) return st;
    StepParams P{};
    P.st = reinterpret_cast<DevState*>(ws);
    LayerW L{};
    for (size_t i = 0; i < M; ++i) {
      GemvArgs a{h->m.view(), p.units, p.upc, x + i * size_t(h->m.K), y + i * size_t(h->m.N), 0};
      CK(launch_k(k_gemv<G_PLAIN>, dim3(p.grid), dim3(kGemvThreads), p.smem, s, false, P, L, a));
    }
    return GAJE_OK;
  }
  if (reinterpret_cast<uintptr_t>(x) & 15u) return set_error(GAJE_ERR_INVALID, "x must be 16-byte aligned");
  if (M >= 16 && h->m.K % kTcK == 0) {  // tensor cores (bf16 hi/lo x3)
    const TcPlan p = tc_plan(h->m.N, h->m.K, int(M), sm_count(h->device));
    const size_t part_b = (p.part_floats * 4 + 255) / 256 * 256;
    const size_t plane = tc_plane_bytes(p.mpad, h->m.K);
    char* ws;
    if (int st = ws_get(h->device, part_b + 2 * plane, &ws, g_ws_tc)) return st;
    TcBuffers tb;
    tb.part = reinterpret_cast<float*>(ws);
    tb.hi = reinterpret_cast<unsigned char*>(ws + part_b);
    tb.lo = tb.hi + plane;
    return tc_gemm_run(p, h->m.tc_rows(), x, int(M), EpiStore{y, h->m.N}, tb, s, false, TcNorm{});
  }
  // 1 < M < 16: every weight word is turned into floats once per CTA for 8
  // vectors; the CTA walks the K splits itself (no workspace)
  constexpr int MT = 8;
  const int ctas = (h->m.N + 2 * kSkWarps - 1) / (2 * kSkWarps);
  const size_t smem = skinny_smem_bytes(MT);
  if (int st = smem_optin((const void*)k_q4_gemm_skinny<MT, false, EpiStore>, smem)) return st;
  k_q4_gemm_skinny<MT, false, EpiStore><<<dim3(ctas, unsigned((M + MT - 1) / MT)), kSkThreads, smem, s>>>(
      h->m.view(), x, int(M), SkNorm{}, SkSplit{}, EpiStore{y, h->m.N});
  CK(cudaGetLastError());
  return GAJE_OK;
}

int gaje_cuda_q4_0_dequant(const gaje_q4_matrix* h, float* w, void* stream) {
  if (!h || !w) return set_error(GAJE_ERR_INVALID, "NULL argument");
  CK(cudaSetDevice(h->device));
  k_dequant_q4<<<1184, 256, 0, (cudaStream_t)stream>>>(h->m.view(), w);
  CK(cudaGetLastError());
  return GAJE_OK;
}

int gaje_cuda_f32_gemv_argmax(const float* W, const float* x, size_t N, size_t K, float* logits, uint32_t* argmax,
                              void* stream) {
  if (!W || !x || !argmax || !N || !K) return set_error(GAJE_ERR_INVALID, "bad argument");
  if (K % 4 || N > 0x7FFFFFFFu || K > (1u << 20)) return set_error(GAJE_ERR_UNSUPPORTED, "K must be a multiple of 4");
  int dev;
  CK(cudaGetDevice(&dev));
  char* ws;
  if (int s = ws_get(dev, kWsAttnBase, &ws)) return s;
  LmArgs a{};
  a.W = W;
  a.x = x;
  a.logits = logits;
  a.N = int(N);
  a.K = int(K);
  const int grid = std::min(sm_count(dev), int(kWsArgmaxParts));
  a.rows_per_cta = int((N + grid - 1) / grid);
  a.stages = lm_stages(int(K));
  if (a.stages < 2) return set_error(GAJE_ERR_UNSUPPORTED, "K too large for the streaming ring");
  a.part = reinterpret_cast<unsigned long long*>(ws + kWsPartsOff);
  a.cnt = reinterpret_cast<unsigned*>(ws + kWsCntOff);
  a.result = argmax;
  const size_t smem = lm_smem_bytes(int(K), a.stages);
  if (int s = smem_optin((const void*)k_lmhead, smem)) return s;
  CK(launch_k(k_lmhead, dim3(grid), dim3(kLmThreads), smem, (cudaStream_t)stream, false, a));
  return GAJE_OK;
}

int gaje_cuda_rms_norm(const float* x, const float* w, float eps, size_t n, float* out, void* stream) {
  if (!x || !w || !out || !n) return set_error(GAJE_ERR_INVALID, "bad argument");
  k_rmsnorm<<<1, 1024, 0, (cudaStream_t)stream>>>(x, w, eps, int(n), out);
  CK(cudaGetLastError());
  return GAJE_OK;
}

}  // extern "C"

// The per-KV-head counters (64 x u32) and timeout marks (64 x u32) ahead of an
// attention call's split partials.
constexpr size_t kAttnScratchHeader = 512;

// Argument checks shared by the two decode-attention entry points, before any
// CUDA call: k_attn bulk-copies cache rows with cp.async.bulk, whose global
// source must be 16-byte aligned, so the caches (and q / out, read and written
// as rows) must be 16-byte aligned and head_dim a multiple of 4.
static int attn_check_args(const float* q, const float* k_cache, const float* v_cache, const float* out, size_t ctx,
                           size_t cache_stride, size_t n_head, size_t n_head_kv, size_t head_dim) {
  if (!q || !k_cache || !v_cache || !out || !ctx || !n_head || !n_head_kv || !head_dim)
    return set_error(GAJE_ERR_INVALID, "bad argument");
  if (((uintptr_t)q | (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)out) & 15u)
    return set_error(GAJE_ERR_INVALID, "q, k_cache, v_cache and out must be 16-byte aligned");
  if (n_head % n_head_kv || n_head / n_head_kv > size_t(kAttnMaxGroup) || ctx > cache_stride || head_dim % 4 ||
      n_head_kv > 64 || cache_stride > (1u << 24))
    return set_error(GAJE_ERR_UNSUPPORTED, "unsupported attention geometry");
  return GAJE_OK;
}

extern "C" {

int gaje_cuda_attention_decode(const float* q, const float* k_cache, const float* v_cache, size_t ctx,
                               size_t cache_stride, size_t n_head, size_t n_head_kv, size_t head_dim, float* out,
                               void* stream) {
  if (int s = attn_check_args(q, k_cache, v_cache, out, ctx, cache_stride, n_head, n_head_kv, head_dim)) return s;
  int dev;
  CK(cudaGetDevice(&dev));
  const size_t G = n_head / n_head_kv;
  const size_t po = n_head_kv * kAttnMaxSplits * G * head_dim, pml = n_head_kv * kAttnMaxSplits * G * 2;
  char* ws;
  if (int s = ws_get(dev, kWsAttnBase + kAttnScratchHeader + (pml + po) * 4 + 256, &ws)) return s;
  char* w = ws + kWsAttnBase;
  AttnArgs a{};
  a.q = q;
  a.kc = k_cache;
  a.vc = v_cache;
  a.out = out;
  a.cnt = reinterpret_cast<unsigned*>(w);
  a.bad = reinterpret_cast<unsigned*>(w + 256);
  a.part_ml = reinterpret_cast<float*>(w + kAttnScratchHeader);
  a.part_o = a.part_ml + pml;
  a.ctx = int(ctx);
  a.stride = int(cache_stride);
  a.nh = int(n_head);
  a.nkv = int(n_head_kv);
  a.hd = int(head_dim);
  a.scale = 1.0f / sqrtf(float(head_dim));
  a.st = nullptr;
  int nsplit, chunk;
  attn_splits(int(ctx), nsplit, chunk);
  const size_t smem = attn_smem_bytes(int(G), int(head_dim), chunk);
  if (int s = smem_optin((const void*)k_attn, smem)) return s;
  CK(launch_k(k_attn, dim3(unsigned(n_head_kv), kAttnMaxSplits), dim3(kAttnThreads), smem, (cudaStream_t)stream,
              false, a));
  return GAJE_OK;
}

// ---- decode attention without allocation
// The same kernel as gaje_cuda_attention_decode with its split partials and
// per-KV-head counters in this file-scope buffer instead of the per-device
// workspace (which is allocated, and re-allocated with a device synchronise
// when a larger geometry arrives).
constexpr size_t kAttnStaticScratchBytes = size_t(1) << 20;  // 1 MiB per device
static __device__ __align__(256) unsigned char g_attn_scratch[kAttnStaticScratchBytes];

int gaje_cuda_attention_decode_static(const float* q, const float* k_cache, const float* v_cache, size_t ctx,
                                      size_t cache_stride, size_t n_head, size_t n_head_kv, size_t head_dim,
                                      float* out, void* stream) {
  if (int s = attn_check_args(q, k_cache, v_cache, out, ctx, cache_stride, n_head, n_head_kv, head_dim)) return s;
  const size_t G = n_head / n_head_kv;
  const size_t po = n_head_kv * kAttnMaxSplits * G * head_dim, pml = n_head_kv * kAttnMaxSplits * G * 2;
  const size_t need = kAttnScratchHeader + (pml + po) * 4;
  if (need > kAttnStaticScratchBytes)
    return set_error(GAJE_ERR_UNSUPPORTED,
                     "attention geometry needs " + std::to_string(need) +
                         " bytes of scratch (512 + n_head*64*(head_dim+2)*4); the static buffer holds " +
                         std::to_string(kAttnStaticScratchBytes));
  int dev;
  CK(cudaGetDevice(&dev));
  // The buffer's device address, looked up with the device current.  The
  // first call on a device does this set-up (it may load the module); later
  // calls look it up again, which allocates nothing and keeps the address
  // valid after the context has been torn down and created again.
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
  if (e != cudaSuccess || !p)
    return set_error(GAJE_ERR_CUDA,
                     std::string("cudaGetSymbolAddress of the attention scratch failed: ") + cudaGetErrorString(e));
  char* w = static_cast<char*>(p);
  AttnArgs a{};
  a.q = q;
  a.kc = k_cache;
  a.vc = v_cache;
  a.out = out;
  // zero at module load; every call, completed or timed out, leaves them zero
  a.cnt = reinterpret_cast<unsigned*>(w);
  a.bad = reinterpret_cast<unsigned*>(w + 256);
  a.part_ml = reinterpret_cast<float*>(w + kAttnScratchHeader);
  a.part_o = a.part_ml + pml;
  a.ctx = int(ctx);
  a.stride = int(cache_stride);
  a.nh = int(n_head);
  a.nkv = int(n_head_kv);
  a.hd = int(head_dim);
  a.scale = 1.0f / sqrtf(float(head_dim));
  a.st = nullptr;
  int nsplit, chunk;
  attn_splits(int(ctx), nsplit, chunk);
  const size_t smem = attn_smem_bytes(int(G), int(head_dim), chunk);
  if (int s = smem_optin((const void*)k_attn, smem)) return s;
  CK(launch_k(k_attn, dim3(unsigned(n_head_kv), kAttnMaxSplits), dim3(kAttnThreads), smem, (cudaStream_t)stream,
              false, a));
  return GAJE_OK;
}

// ---- quantisers on the device (quant.cuh)
static int quantize_device(const float* w, size_t n, uint8_t* out, void* stream, bool q8) {
  if (!w || !out) return set_error(GAJE_ERR_INVALID, "NULL pointer");
  if (n % 32) return set_error(GAJE_ERR_INVALID, "Weights length must be divisible by 32");
  if ((uintptr_t)w & 15u) return set_error(GAJE_ERR_INVALID, "w must be 16-byte aligned");
  if ((uintptr_t)out & (q8 ? 1u : 3u))
    return set_error(GAJE_ERR_INVALID, q8 ? "out must be 2-byte aligned" : "out must be 4-byte aligned");
  const size_t nblocks = n / 32;
  if (!nblocks) return GAJE_OK;
  int dev;
  CK(cudaGetDevice(&dev));
  const size_t tiles = (nblocks + kQuantThreads - 1) / kQuantThreads;
  const unsigned grid = unsigned(std::min<size_t>(tiles, size_t(sm_count(dev)) * 6));
  if (q8)
    k_quantize_q8_0<<<grid, kQuantThreads, 0, (cudaStream_t)stream>>>(w, nblocks, out);
  else
    k_quantize_q4_0<<<grid, kQuantThreads, 0, (cudaStream_t)stream>>>(w, nblocks, out);
  CK(cudaGetLastError());
  return GAJE_OK;
}

int gaje_cuda_sample_top_p(const float* logits, size_t n, float temperature, float top_p, float r, uint32_t* token,
                           uint32_t* kept, void* stream) {
  if (!logits || !token) return set_error(GAJE_ERR_INVALID, "NULL argument");
  if (n > (size_t(1) << 23)) return set_error(GAJE_ERR_INVALID, "n above 2^23");
  if (!(temperature > 0.0f) || !(r >= 0.0f && r < 1.0f) || top_p != top_p)
    return set_error(GAJE_ERR_INVALID, "temperature must be > 0, r in [0, 1), top_p a number");
  k_sample_top_p<<<1, kSampleThreads, 0, (cudaStream_t)stream>>>(logits, int(n), temperature, top_p, r, token, kept);
  CK(cudaGetLastError());
  return GAJE_OK;
}

int gaje_cuda_quantize_q4_0(const float* w, size_t n, uint8_t* out, void* stream) {
  return quantize_device(w, n, out, stream, false);
}

int gaje_cuda_quantize_q8_0(const float* w, size_t n, uint8_t* out, void* stream) {
  return quantize_device(w, n, out, stream, true);
}

int gaje_cuda_kwta(float* scores, size_t n, size_t k, void* stream) {
  if (!scores) return set_error(GAJE_ERR_INVALID, "scores is NULL");
  if (n > 0x7FFFFFFFu) return set_error(GAJE_ERR_INVALID, "n too large");
  k_kwta<<<1, kKwtaThreads, 0, (cudaStream_t)stream>>>(scores, int(n), int(std::min<size_t>(k, 0x7FFFFFFF)));
  CK(cudaGetLastError());
  return GAJE_OK;
}

}  // extern "C"
