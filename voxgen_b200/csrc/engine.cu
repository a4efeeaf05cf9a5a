// C ABI of the B200 BaseLM decode step (include/voxgen_cuda.h).
//
// Host side of the hot path: replaces BaseLmEngine (src/baselm.rs:429-1232)
// and the Vulkan dispatch it records into (src/vulkan.rs). A decode step is
// one cooperative launch of the persistent step kernel (step_kernel.cuh: every
// layer's phases in one launch, grid barriers between them), captured in a
// CUDA graph per step variant. Position, token and error flags live in a
// device control block, so one instantiated graph replays every step. Streams
// whose model the persistent kernel does not take (projections in two weight
// formats, no cooperative launch, or VOXGEN_STEP_KERNEL=0) run the step as a
// program of one launch per projection / attention / norm (build_program),
// chained with programmatic dependent launch and captured the same way.
#include <cuda_runtime.h>
#include <sys/mman.h>
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "../../include/voxgen_cuda.h"
#include "gguf_loader.h"
#include "batch_kernel.cuh"

using namespace vg;

// ---------------------------------------------------------------------------
// handles
// ---------------------------------------------------------------------------
struct vg_ctx {
  int device = 0;
  int sms = 0;
  std::string err;
  std::mutex mu;
};

namespace {

struct DevMat {
  uint8_t *w = nullptr;
  TileGeom g{0, 0, 1};
  uint32_t type = GGML_Q8_0;
};

DevMat make_mat(uint32_t rows, uint32_t cols, uint32_t type) {
  DevMat d;
  d.g = TileGeom{rows, cols, type == GGML_Q8_0 ? 1u : 0u};
  d.type = type;
  return d;
}

struct Layer {
  DevMat qkv, o, gateup, down;
  float *attn_norm = nullptr, *ffn_norm = nullptr;
};

struct Launch {
  std::function<cudaError_t(cudaStream_t, bool)> fn;
  const char *name = "";
  uint32_t layer = 0;
  uint64_t bytes = 0;    // algorithmic HBM bytes (attention: per KV row, scaled at run time)
  bool per_position = false;
};

constexpr uint32_t kStagingSlots = 16;
constexpr uint32_t kSmemBudget = 112 * 1024;  // per matvec CTA: two kernels share an SM under PDL
constexpr uint32_t kSmemMax = 227 * 1024;

std::mutex g_live_mu;
std::set<const void *> g_live;

void live_add(const void *p) {
  std::lock_guard<std::mutex> l(g_live_mu);
  g_live.insert(p);
}
void live_del(const void *p) {
  std::lock_guard<std::mutex> l(g_live_mu);
  g_live.erase(p);
}
bool live(const void *p) {
  std::lock_guard<std::mutex> l(g_live_mu);
  return p && g_live.count(p);
}

std::string strf(const char *f, ...) __attribute__((format(printf, 1, 2)));
std::string strf(const char *f, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof buf, f, ap);
  va_end(ap);
  return buf;
}

[[noreturn]] void fail(int code, const std::string &m) { throw Error{code, m}; }

#define CK(call)                                                                               \
  do {                                                                                         \
    cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess)                                                                     \
      fail(e_ == cudaErrorMemoryAllocation ? VG_ENOMEM : VG_ECUDA,                             \
           strf("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__)); \
  } while (0)

uint32_t round_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }
size_t round_up_sz(size_t x, size_t a) { return (x + a - 1) / a * a; }

uint64_t packed_bytes(uint32_t type, uint32_t rows, uint32_t cols) {
  return TileGeom{rows, cols, type == GGML_Q8_0 ? 1u : 0u}.bytes();
}

// Test hook (vg_test_fake_event_status): when nonzero, host_wait treats every
// event query as having returned this status, as a driver would report a
// kernel that timed out (cudaErrorLaunchTimeout); the GPU work is untouched.
std::atomic<int> g_fake_event_status{0};

// Bounded host wait on an event: spin briefly, then poll with short sleeps.
int host_wait(cudaEvent_t ev, uint64_t timeout_ns) {
  const auto t0 = std::chrono::steady_clock::now();
  for (uint64_t it = 0;; ++it) {
    const int fake = g_fake_event_status.load(std::memory_order_relaxed);
    cudaError_t e = fake ? (cudaError_t)fake : cudaEventQuery(ev);
    if (e == cudaSuccess) return VG_OK;
    if (e != cudaErrorNotReady) fail(VG_ECUDA, strf("cudaEventQuery failed: %s", cudaGetErrorString(e)));
    const uint64_t el = (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                            std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_ns) return VG_ETIMEDOUT;
    if (el > 2000000) std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

template <class K, class... Args>
cudaError_t launch_ex(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, uint32_t cluster_x,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = n ? attr : nullptr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---- matvec planning --------------------------------------------------------
using MvFn = void (*)(MvParams);

template <Mode M, Pro P>
MvFn matvec_fn(bool q8) {
  return q8 ? matvec_kernel<true, M, P> : matvec_kernel<false, M, P>;
}

std::mutex g_attr_mu;
std::map<std::pair<int, const void *>, int> g_smem_attr;  // (device, fn) -> bytes set

void ensure_smem(const void *fn, int device, uint32_t bytes) {
  std::lock_guard<std::mutex> l(g_attr_mu);
  int &cur = g_smem_attr[{device, fn}];
  if ((int)bytes > cur) {
    CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    cur = (int)bytes;
  }
}

struct MvPlan {
  MvFn fn = nullptr;
  dim3 grid;
  uint32_t smem = 0;
  MvParams p{};
};

template <Mode M, Pro P>
MvPlan plan_matvec(const DevMat &m, int device, uint32_t sms) {
  MvPlan pl;
  const TileGeom g = m.g;
  const uint32_t T = g.tiles();
  const uint32_t grid = std::min<uint32_t>(sms, T);
  const uint32_t per_cta = (T + grid - 1) / grid;
  const uint32_t cols_pad = g.nseg() * g.seg_cols();
  MvParams &p = pl.p;
  p.w = m.w;
  p.g = g;
  p.a_bytes = mv_a_bytes(g.q8, cols_pad);
  p.plane = mv_a_plane(g.q8, cols_pad);
  // One partial-sum row per tile of the CTA.
  p.rb = per_cta;
  // Pipeline stages: as many as the budget holds (up to 8), at most the CTA's
  // stage count, at least 2 so a copy is in flight while a stage is consumed.
  const uint32_t n_st = (per_cta * g.nseg() + kStageSegs - 1) / kStageSegs;
  p.stages = 1;
  MvSmem probe(p);
  const uint32_t per_stage = kStageSegs * g.seg_bytes() + 16u;
  const uint32_t fixed = probe.total - per_stage;
  const uint32_t fit = kSmemBudget > fixed ? (kSmemBudget - fixed) / per_stage : 1u;
  const uint32_t st = std::min<uint32_t>({fit, 8u, std::max<uint32_t>(2u, n_st)});
  if (st < 2) fail(VG_EUNSUPPORTED, strf("matrix of %u columns does not fit two pipeline stages", g.cols));
  p.stages = st;
  const uint32_t smem = MvSmem(p).total;
  if (smem > kSmemMax) fail(VG_EUNSUPPORTED, strf("matrix of %u columns does not fit in shared memory", g.cols));
  pl.fn = matvec_fn<M, P>(g.q8 != 0);
  pl.grid = dim3(grid);
  pl.smem = smem;
  ensure_smem((const void *)pl.fn, device, smem);
  return pl;
}

cudaError_t run_matvec(const MvPlan &pl, cudaStream_t st, bool pdl) {
  return launch_ex(pl.fn, pl.grid, dim3(kMvThreads), pl.smem, st, pdl, 1u, pl.p);
}

// Attention split count: chunks of at most 64 positions, a multiple of the cluster size.
void plan_attention(uint32_t ctx, uint32_t &nsplit, uint32_t &chunk_cap) {
  nsplit = std::max<uint32_t>(1u, (ctx + 63u) / 64u);
  nsplit = (nsplit + kAttnCluster - 1) / kAttnCluster * kAttnCluster;
  chunk_cap = (ctx + nsplit - 1) / nsplit;
}

using AttnFn = void (*)(AttnParams);
AttnFn pick_attention(uint32_t head_dim) {
  switch (head_dim) {
    case 32: return attention_kernel<1>;
    case 64: return attention_kernel<2>;
    case 128: return attention_kernel<4>;
    default: return attention_kernel<8>;
  }
}

}  // namespace

// Plan and workspace of decode_batch_kernel (batch_kernel.cuh) for one model,
// made at the first vg_decode_batch / vg_prefill_tokens that can use it.
constexpr uint32_t kBatchStaging = 4;  // pinned slots of column tables in flight

struct BatchWork {
  std::string why;  // why the batched kernel is unavailable for this model ("": available)
  BatchParams p{};
  void (*fn)(BatchParams) = nullptr;
  uint32_t smem = 0, grid = 0;
  void *dev = nullptr;            // device workspace
  uint8_t *pin = nullptr;         // kBatchStaging x (column table + control block)
  size_t pin_stride = 0, table_bytes = 0;
  cudaEvent_t pin_ev[kBatchStaging] = {};
  uint32_t pin_next = 0;
  cudaStream_t st = nullptr;      // every launch of the model's batched kernel goes here
  cudaEvent_t ev_done = nullptr;
};

struct vg_model {
  vg_ctx *ctx = nullptr;
  BaseLmConfig cfg;
  GgufSummary summary;
  uint8_t *arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<Layer> layers;
  DevMat tok, out;
  float *out_norm = nullptr, *inv_freq = nullptr, *ext = nullptr;
  bool rope_ok = true;
  vg_model_info info{};
  int streams = 0;
  // ResidualLM + FSQ + fusion of an acoustic GGUF (vg_residual_load_gguf):
  // the layers above, no token table or LM head, no RoPE
  bool residual = false;
  AcousticConfig acoustic;
  DevMat fsq_in, fsq_out, fuse;  // [latent x H], [H x latent], [H x 2H]
  float *fsq_in_b = nullptr, *fsq_out_b = nullptr, *fuse_b = nullptr;
  // workspace of the batched step kernel (vg_decode_batch, vg_prefill_tokens),
  // made at first use; batch_mu serialises its use by host threads
  BatchWork *batch = nullptr;
  std::mutex batch_mu;
};

struct vg_stream {
  vg_model *m = nullptr;
  uint32_t max_ctx = 0, pos = 0, nsplit = 0, chunk_cap = 0;
  cudaStream_t st = nullptr;
  __half *kc = nullptr, *vc = nullptr;  // [layer][kv_head][max_ctx][head_dim]
  float *hid_a = nullptr, *hid_b = nullptr, *q = nullptr, *attn = nullptr, *gate = nullptr;
  float *out_norm = nullptr, *logits = nullptr, *part = nullptr;
  uint32_t *tickets = nullptr, *ctrl = nullptr;
  void *dev_block = nullptr;
  // pinned staging: kStagingSlots x (token + H floats), and the output block
  uint8_t *pin_in = nullptr;
  size_t pin_in_stride = 0;
  cudaEvent_t pin_ev[kStagingSlots] = {};
  uint32_t pin_next = 0;
  uint8_t *pin_out = nullptr;
  cudaEvent_t ev_done = nullptr;
  cudaGraphExec_t graphs[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};  // [token_input][logits]
  bool logits_valid = false;
  // persistent decode-step kernel (one cooperative launch per token)
  bool use_step = false;     // else the step is the per-kernel program of build_program
  bool step_graph = true;    // the cooperative launch is captured in the step graphs
  StepParams sp{};           // token_input / want_logits set per launch
  void (*step_fn)(StepParams) = nullptr;
  uint32_t step_smem = 0, step_grid = 0;
  bool step_head_apart = false;  // the LM head is stored in another format: own launch after the step
  MvPlan step_head{};
  // ResidualLM streams: the BaseLM hidden state in (FSQ positions), the FSQ
  // latent, the FSQ output, the fusion input [LM state | acoustic embedding]
  // (the LM state is the FSQ output or the raw BaseLM hidden), the fusion
  // output (snapshot), and the three matvec plans of the per-kernel path
  float *res_base = nullptr, *fsq_lat = nullptr, *fsq_res = nullptr, *fuse_in = nullptr, *fused = nullptr;
  MvPlan fsq_in_p{}, fsq_out_p{}, fuse_p{};
  // the LM head as its own launch on the output (logits after a batched prefill)
  MvPlan head_plan{};
  bool head_planned = false;
};

namespace {

void set_err(vg_ctx *c, const std::string &msg) {
  if (!c) return;
  std::lock_guard<std::mutex> l(c->mu);
  c->err = msg;
}

template <class F>
int guard(vg_ctx *c, F &&f) {
  try {
    return f();
  } catch (const Error &e) {
    set_err(c, e.msg);
    return e.code;
  } catch (const std::bad_alloc &) {
    set_err(c, "host allocation failed");
    return VG_ENOMEM;
  } catch (const std::exception &e) {
    set_err(c, e.what());
    return VG_EINVAL;
  }
}

void fill_info(vg_model *m) {
  const BaseLmConfig &c = m->cfg;
  vg_model_info &i = m->info;
  i.context_length = c.context_length;
  i.embedding_length = c.embedding_length;
  i.block_count = c.block_count;
  i.feed_forward_length = c.feed_forward_length;
  i.vocab_size = c.vocab_size;
  i.head_count = c.head_count;
  i.head_count_kv = c.head_count_kv;
  i.head_dim = c.head_dim;
  i.kv_dim = c.kv_dim;
  i.rope_original_context_length = c.rope_original_context_length;
  i.rms_epsilon = c.rms_epsilon;
  i.rope_theta = c.rope_theta;
  i.rope_scaling_factor = c.rope_scaling_factor();
  i.embedding_scale = c.embedding_scale;
  i.residual_scale = c.residual_scale;
  i.logit_scale = c.logit_scale;
  i.format = (int32_t)c.format;
  i.tied_output = c.tied_output;
  i.rope_long_factors = c.rope_scaling_type == "longrope" && c.rope_long();
  i.gguf_data_bytes = m->summary.file_bytes - m->summary.data_offset;
  uint64_t lw = 0;
  for (uint32_t l = 0; l < c.block_count; ++l)
    for (const char *s : {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"})
      lw += m->summary.find(strf(m->residual ? "residual_lm.blk.%u.%s.weight" : "blk.%u.%s.weight", l, s))->bytes;
  i.layer_weight_bytes = lw;
  i.norm_weight_bytes = (uint64_t)(2 * c.block_count + 1) * c.embedding_length * 4;
  i.device_weight_bytes = m->arena_bytes;
}

float eff_scale(float v) { return v == 0.0f ? 1.0f : v; }  // effective_scale, src/baselm.rs:1262-1264

void load_model(vg_model *m, const std::string &path, uint32_t requested) {
  m->summary = load_summary(path);
  m->cfg = config_from_gguf(m->summary, requested);
  check_kernel_support(m->summary, m->cfg);
  const BaseLmConfig &c = m->cfg;
  const GgufSummary &S = m->summary;
  const uint32_t H = c.embedding_length, F = c.feed_forward_length, KV = c.kv_dim;

  // ---- arena layout ----
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = round_up_sz(off + bytes, 256);
    return o;
  };
  struct Pending {
    DevMat *mat;
    size_t off;
  };
  std::vector<Pending> mats;
  std::vector<std::pair<float **, size_t>> vecs;
  m->layers.resize(c.block_count);
  auto tensor = [&](const std::string &n) -> const TensorInfo & { return *S.find(n); };
  for (uint32_t l = 0; l < c.block_count; ++l) {
    Layer &L = m->layers[l];
    auto nm = [&](const char *s) { return strf("blk.%u.%s.weight", l, s); };
    const uint32_t tq = tensor(nm("attn_q")).type, to = tensor(nm("attn_output")).type;
    const uint32_t tg = tensor(nm("ffn_gate")).type, td = tensor(nm("ffn_down")).type;
    L.qkv = make_mat(H + 2 * KV, H, tq);
    L.o = make_mat(H, H, to);
    L.gateup = make_mat(2 * F, H, tg);
    L.down = make_mat(H, F, td);
    for (DevMat *d : {&L.qkv, &L.o, &L.gateup, &L.down}) mats.push_back({d, take(d->g.bytes())});
    vecs.push_back({&L.attn_norm, take((size_t)H * 4)});
    vecs.push_back({&L.ffn_norm, take((size_t)H * 4)});
  }
  const TensorInfo &tok = tensor("token_embd.weight");
  m->tok = make_mat(c.vocab_size, H, tok.type);
  mats.push_back({&m->tok, take(m->tok.g.bytes())});
  if (!c.tied_output) {
    const TensorInfo &o = tensor("output.weight");
    m->out = make_mat(c.vocab_size, H, o.type);
    mats.push_back({&m->out, take(m->out.g.bytes())});
  }
  vecs.push_back({&m->out_norm, take((size_t)H * 4)});
  vecs.push_back({&m->inv_freq, take((size_t)c.head_dim / 2 * 4)});
  vecs.push_back({&m->ext, take((size_t)c.head_dim / 2 * 4)});
  m->arena_bytes = off;
  CK(cudaMalloc(&m->arena, m->arena_bytes));
  for (auto &p : mats) p.mat->w = m->arena + p.off;
  CK(cudaMemset(m->arena, 0, m->arena_bytes));  // tile padding stays zero
  for (auto &v : vecs) *v.first = reinterpret_cast<float *>(m->arena + v.second);
  if (c.tied_output) m->out = m->tok;

  // ---- upload + repack ----
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) fail(VG_EIO, "open " + path + " failed");
  void *map = mmap(nullptr, S.file_bytes, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map == MAP_FAILED) fail(VG_EIO, "mmap " + path + " failed");
  const uint8_t *data = static_cast<const uint8_t *>(map) + S.data_offset;
  size_t max_raw = 0;
  for (const auto &t : S.tensors) max_raw = std::max<size_t>(max_raw, t.bytes);
  uint8_t *staging = nullptr;
  cudaStream_t st = nullptr;
  try {
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    CK(cudaMalloc(&staging, max_raw));
    // row0: first packed row of this tensor inside dst (a multiple of the tile height)
    auto repack = [&](const std::string &name, const DevMat &dst, uint32_t row0, uint32_t perm, uint32_t group,
                      uint32_t half) {
      const TensorInfo &t = tensor(name);
      CK(cudaMemcpyAsync(staging, data + t.offset, t.bytes, cudaMemcpyHostToDevice, st));
      const uint32_t rows = (uint32_t)t.dims[1];
      if (row0 % kTileRows) fail(VG_EUNSUPPORTED, "tensor " + name + " does not start on a tile boundary");
      TileGeom sub = dst.g;  // the tensor's rows as their own tiled matrix inside dst
      sub.rows = dst.g.rows - row0;
      repack_kernel<<<std::min<uint32_t>(rows, 65535u), 256, 0, st>>>(
          staging, rows, sub, dst.w + dst.g.seg_base(row0, 0), perm, group, half);
      CK(cudaGetLastError());
      CK(cudaStreamSynchronize(st));
    };
    auto upload_vec = [&](const std::string &name, float *dst) {
      const TensorInfo &t = tensor(name);
      CK(cudaMemcpy(dst, data + t.offset, t.bytes, cudaMemcpyHostToDevice));
    };
    for (uint32_t l = 0; l < c.block_count; ++l) {
      Layer &L = m->layers[l];
      auto nm = [&](const char *s) { return strf("blk.%u.%s.weight", l, s); };
      repack(nm("attn_q"), L.qkv, 0, kPermRope, c.head_dim, 0);
      repack(nm("attn_k"), L.qkv, H, kPermRope, c.head_dim, 0);
      repack(nm("attn_v"), L.qkv, H + KV, kPermIdentity, 0, 0);
      repack(nm("attn_output"), L.o, 0, kPermIdentity, 0, 0);
      repack(nm("ffn_gate"), L.gateup, 0, kPermHalves, 0, 0);
      repack(nm("ffn_up"), L.gateup, 0, kPermHalves, 0, 1);
      repack(nm("ffn_down"), L.down, 0, kPermIdentity, 0, 0);
      upload_vec(nm("attn_norm"), L.attn_norm);
      upload_vec(nm("ffn_norm"), L.ffn_norm);
    }
    repack("token_embd.weight", m->tok, 0, kPermIdentity, 0, 0);
    if (!c.tied_output) repack("output.weight", m->out, 0, kPermIdentity, 0, 0);
    upload_vec("output_norm.weight", m->out_norm);
    // RoPE tables: inv_freq as rope.comp:29-30 computes it, evaluated once on
    // the host; ext = the factor set record_transformer picks (baselm.rs:902-913).
    std::vector<float> inv(c.head_dim / 2), ext(c.head_dim / 2, 1.0f);
    for (uint32_t i = 0; i < c.head_dim / 2; ++i)
      inv[i] = 1.0f / powf(c.rope_theta, (float)(i * 2u) / (float)c.head_dim);
    m->rope_ok = c.rope_scaling_type == "longrope";
    if (m->rope_ok) {
      const TensorInfo &f = tensor(c.rope_long() ? "rope_factors_long.weight" : "rope_factors_short.weight");
      std::memcpy(ext.data(), data + f.offset, ext.size() * 4);
    }
    CK(cudaMemcpy(m->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(m->ext, ext.data(), ext.size() * 4, cudaMemcpyHostToDevice));
  } catch (...) {
    munmap(map, S.file_bytes);
    if (staging) cudaFree(staging);
    if (st) cudaStreamDestroy(st);
    throw;
  }
  munmap(map, S.file_bytes);
  cudaFree(staging);
  cudaStreamDestroy(st);
  fill_info(m);
}

// The ResidualLM + FSQ + fusion part of an acoustic GGUF
// (ResidualFsqEngine::new, src/acoustic.rs:435-560), following the BaseLM
// model base: its layers are repacked exactly like the BaseLM's, the step
// kernel runs them with RoPE off (inv_freq = 0 makes the rotation (1, 0)),
// and FSQ and the fusion projection are matvecs with the bias as residual.
void load_residual_model(vg_model *m, const std::string &path, const vg_model *base) {
  m->summary = load_summary(path);
  const GgufSummary &S = m->summary;
  m->acoustic = acoustic_from_gguf(S, base->cfg);
  m->residual = true;
  BaseLmConfig c = base->cfg;
  c.block_count = m->acoustic.residual_block_count;
  c.vocab_size = 0;
  c.context_length = 8192;  // VOXCPM2_MAX_GENERATION_CONTEXT, src/acoustic.rs:72-76
  c.rope_scaling_type = "none";
  c.format = GGML_F16;
  c.tied_output = true;
  c.output_tensor.clear();
  m->cfg = c;
  const uint32_t H = c.embedding_length, F = c.feed_forward_length, KV = c.kv_dim;
  const uint32_t QR = c.head_count * c.head_dim, LAT = m->acoustic.fsq_latent_dim;
  auto tensor = [&](const std::string &n) -> const TensorInfo & { return *S.find(n); };
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = round_up_sz(off + bytes, 256);
    return o;
  };
  struct Pending {
    DevMat *mat;
    size_t off;
  };
  std::vector<Pending> mats;
  std::vector<std::pair<float **, size_t>> vecs;
  m->layers.resize(c.block_count);
  for (uint32_t l = 0; l < c.block_count; ++l) {
    Layer &L = m->layers[l];
    L.qkv = make_mat(QR + 2 * KV, H, GGML_F16);
    L.o = make_mat(H, QR, GGML_F16);
    L.gateup = make_mat(2 * F, H, GGML_F16);
    L.down = make_mat(H, F, GGML_F16);
    for (DevMat *d : {&L.qkv, &L.o, &L.gateup, &L.down}) mats.push_back({d, take(d->g.bytes())});
    vecs.push_back({&L.attn_norm, take((size_t)H * 4)});
    vecs.push_back({&L.ffn_norm, take((size_t)H * 4)});
  }
  m->fsq_in = make_mat(LAT, H, GGML_F16);
  m->fsq_out = make_mat(H, LAT, GGML_F16);
  m->fuse = make_mat(H, 2 * H, GGML_F16);
  for (DevMat *d : {&m->fsq_in, &m->fsq_out, &m->fuse}) mats.push_back({d, take(d->g.bytes())});
  vecs.push_back({&m->fsq_in_b, take((size_t)LAT * 4)});
  vecs.push_back({&m->fsq_out_b, take((size_t)H * 4)});
  vecs.push_back({&m->fuse_b, take((size_t)H * 4)});
  vecs.push_back({&m->out_norm, take((size_t)H * 4)});
  vecs.push_back({&m->inv_freq, take((size_t)c.head_dim / 2 * 4)});
  vecs.push_back({&m->ext, take((size_t)c.head_dim / 2 * 4)});
  m->arena_bytes = off;
  CK(cudaMalloc(&m->arena, m->arena_bytes));
  for (auto &p : mats) p.mat->w = m->arena + p.off;
  CK(cudaMemset(m->arena, 0, m->arena_bytes));  // tile padding stays zero
  for (auto &v : vecs) *v.first = reinterpret_cast<float *>(m->arena + v.second);

  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) fail(VG_EIO, "open " + path + " failed");
  void *map = mmap(nullptr, S.file_bytes, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map == MAP_FAILED) fail(VG_EIO, "mmap " + path + " failed");
  const uint8_t *data = static_cast<const uint8_t *>(map) + S.data_offset;
  size_t max_raw = 0;
  for (const auto &t : S.tensors) max_raw = std::max<size_t>(max_raw, t.bytes);
  uint8_t *staging = nullptr;
  cudaStream_t st = nullptr;
  try {
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    CK(cudaMalloc(&staging, max_raw));
    auto repack = [&](const std::string &name, const DevMat &dst, uint32_t row0, uint32_t perm, uint32_t group,
                      uint32_t half) {
      const TensorInfo &t = tensor(name);
      CK(cudaMemcpyAsync(staging, data + t.offset, t.bytes, cudaMemcpyHostToDevice, st));
      const uint32_t rows = (uint32_t)t.dims[1];
      if (row0 % kTileRows) fail(VG_EUNSUPPORTED, "tensor " + name + " does not start on a tile boundary");
      TileGeom sub = dst.g;
      sub.rows = dst.g.rows - row0;
      repack_kernel<<<std::min<uint32_t>(rows, 65535u), 256, 0, st>>>(
          staging, rows, sub, dst.w + dst.g.seg_base(row0, 0), perm, group, half);
      CK(cudaGetLastError());
      CK(cudaStreamSynchronize(st));
    };
    // vectors as fp32 (the biases may be stored F16: load_scalar, linear_bias.comp)
    auto upload_vec = [&](const std::string &name, float *dst) {
      const TensorInfo &t = tensor(name);
      std::vector<float> v(t.elements);
      for (uint64_t i = 0; i < t.elements; ++i)
        v[i] = t.type == GGML_F32 ? reinterpret_cast<const float *>(data + t.offset)[i]
                                  : __half2float(reinterpret_cast<const __half *>(data + t.offset)[i]);
      CK(cudaMemcpy(dst, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
    };
    for (uint32_t l = 0; l < c.block_count; ++l) {
      Layer &L = m->layers[l];
      auto nm = [&](const char *x) { return strf("residual_lm.blk.%u.%s.weight", l, x); };
      repack(nm("attn_q"), L.qkv, 0, kPermRope, c.head_dim, 0);
      repack(nm("attn_k"), L.qkv, QR, kPermRope, c.head_dim, 0);
      repack(nm("attn_v"), L.qkv, QR + KV, kPermIdentity, 0, 0);
      repack(nm("attn_output"), L.o, 0, kPermIdentity, 0, 0);
      repack(nm("ffn_gate"), L.gateup, 0, kPermHalves, 0, 0);
      repack(nm("ffn_up"), L.gateup, 0, kPermHalves, 0, 1);
      repack(nm("ffn_down"), L.down, 0, kPermIdentity, 0, 0);
      upload_vec(nm("attn_norm"), L.attn_norm);
      upload_vec(nm("ffn_norm"), L.ffn_norm);
    }
    repack("fsq.in_proj.weight", m->fsq_in, 0, kPermIdentity, 0, 0);
    repack("fsq.out_proj.weight", m->fsq_out, 0, kPermIdentity, 0, 0);
    repack("projections.res_fusion_proj.weight", m->fuse, 0, kPermIdentity, 0, 0);
    upload_vec("fsq.in_proj.bias", m->fsq_in_b);
    upload_vec("fsq.out_proj.bias", m->fsq_out_b);
    upload_vec("projections.res_fusion_proj.bias", m->fuse_b);
    upload_vec("residual_lm.output_norm.weight", m->out_norm);
    // no RoPE (record_residual_lm, src/acoustic.rs:968-970): angle 0, factor 1
    std::vector<float> inv(c.head_dim / 2, 0.0f), ext(c.head_dim / 2, 1.0f);
    CK(cudaMemcpy(m->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(m->ext, ext.data(), ext.size() * 4, cudaMemcpyHostToDevice));
    m->rope_ok = true;
  } catch (...) {
    munmap(map, S.file_bytes);
    if (staging) cudaFree(staging);
    if (st) cudaStreamDestroy(st);
    throw;
  }
  munmap(map, S.file_bytes);
  cudaFree(staging);
  cudaStreamDestroy(st);
  fill_info(m);
}

// ---- step recording ---------------------------------------------------------
// GGUF bytes of one matrix row of `cols` columns (the algorithmic bytes read).
uint64_t gguf_bytes(uint32_t type, uint32_t cols) {
  return type == GGML_Q8_0 ? (uint64_t)cols / 32 * 34 : (uint64_t)cols * 2;
}

void build_program(vg_stream *s, bool token_input, bool logits, std::vector<Launch> &prog) {
  vg_model *m = s->m;
  const BaseLmConfig &c = m->cfg;
  const int dev = m->ctx->device;
  const uint32_t sms = (uint32_t)m->ctx->sms;
  const uint32_t H = c.embedding_length, D = c.head_dim, G = c.head_count / c.head_count_kv;
  const float rs = eff_scale(c.residual_scale);
  uint32_t *ctrl = s->ctrl;
  if (token_input) {
    const DevMat tok = m->tok;
    const float alpha = eff_scale(c.embedding_scale);
    float *out = s->hid_a;
    prog.push_back({[=](cudaStream_t st, bool pdl) {
      return launch_ex(embedding_kernel, dim3((H + 255) / 256), dim3(256), 0, st, pdl, 1u, (const uint8_t *)tok.w,
                       tok.g, (const uint32_t *)(ctrl + kCtrlToken), 0u, alpha, out, ctrl + kCtrlErr);
    }, "embedding", 0, gguf_bytes(tok.type, H)});
  }
  const AttnFn afn = pick_attention(D);
  const uint32_t asmem = attention_smem_bytes(G, D, s->chunk_cap);
  ensure_smem((const void *)afn, dev, asmem);
  for (uint32_t l = 0; l < c.block_count; ++l) {
    const Layer &L = m->layers[l];
    __half *kc = s->kc + (size_t)l * c.head_count_kv * s->max_ctx * D;
    __half *vc = s->vc + (size_t)l * c.head_count_kv * s->max_ctx * D;
    MvPlan qkv = plan_matvec<Mode::QKV, Pro::RMSNORM>(L.qkv, dev, sms);
    qkv.p.xsrc = s->hid_a;
    qkv.p.normw = L.attn_norm;
    qkv.p.eps = c.rms_epsilon;
    qkv.p.out = s->q;
    qkv.p.q_rows = H;
    qkv.p.kv_rows = c.kv_dim;
    qkv.p.head_dim = D;
    qkv.p.ctx = s->max_ctx;
    qkv.p.kc = kc;
    qkv.p.vc = vc;
    qkv.p.inv_freq = m->inv_freq;
    qkv.p.ext = m->ext;
    qkv.p.rope_scaling = c.rope_scaling_factor();
    qkv.p.ctrl = ctrl;
    prog.push_back({[=](cudaStream_t st, bool pdl) { return run_matvec(qkv, st, pdl); }, "qkv", l,
                    gguf_bytes(L.qkv.type, H) * L.qkv.g.rows + (uint64_t)H * 4 + 2ull * c.kv_dim * 2});

    AttnParams ap{};
    ap.q = s->q;
    ap.kc = kc;
    ap.vc = vc;
    ap.out = s->attn;
    ap.part = s->part;
    ap.tickets = s->tickets;
    ap.heads = c.head_count;
    ap.kv_heads = c.head_count_kv;
    ap.ctx = s->max_ctx;
    ap.nsplit = s->nsplit;
    ap.chunk_cap = s->chunk_cap;
    ap.scale = 1.0f / sqrtf((float)D);
    ap.fixed_pos = 0xFFFFFFFFu;
    ap.ctrl = ctrl;
    ap.swz = 1;  // the stream's cache holds chunk-permuted rows (kv_swz)
    prog.push_back({[=](cudaStream_t st, bool pdl) {
      return launch_ex(afn, dim3(ap.nsplit, ap.kv_heads), dim3(kAttnThreads), asmem, st, pdl, kAttnCluster, ap);
    }, "attention", l, 2ull * c.kv_dim * 2, true});

    MvPlan o = plan_matvec<Mode::RESID, Pro::COPY>(L.o, dev, sms);
    o.p.xsrc = s->attn;
    o.p.out = s->hid_b;
    o.p.resid = s->hid_a;
    o.p.alpha = rs;
    o.p.ctrl = ctrl;
    prog.push_back({[=](cudaStream_t st, bool pdl) { return run_matvec(o, st, pdl); }, "o_proj", l,
                    gguf_bytes(L.o.type, H) * L.o.g.rows});

    MvPlan gu = plan_matvec<Mode::SWIGLU, Pro::RMSNORM>(L.gateup, dev, sms);
    gu.p.xsrc = s->hid_b;
    gu.p.normw = L.ffn_norm;
    gu.p.eps = c.rms_epsilon;
    gu.p.out = s->gate;
    gu.p.ctrl = ctrl;
    prog.push_back({[=](cudaStream_t st, bool pdl) { return run_matvec(gu, st, pdl); }, "gate_up", l,
                    gguf_bytes(L.gateup.type, H) * L.gateup.g.rows + (uint64_t)H * 4});

    MvPlan dn = plan_matvec<Mode::RESID, Pro::COPY>(L.down, dev, sms);
    dn.p.xsrc = s->gate;
    dn.p.out = s->hid_a;
    dn.p.resid = s->hid_b;
    dn.p.alpha = rs;
    dn.p.ctrl = ctrl;
    prog.push_back({[=](cudaStream_t st, bool pdl) { return run_matvec(dn, st, pdl); }, "down", l,
                    gguf_bytes(L.down.type, c.feed_forward_length) * L.down.g.rows});
  }
  {
    float *hid = s->hid_a, *y = s->out_norm;
    const float *w = m->out_norm;
    const float eps = c.rms_epsilon;
    prog.push_back({[=](cudaStream_t st, bool pdl) {
      return launch_ex(residual_rmsnorm_kernel, dim3(1), dim3(std::min<uint32_t>(1024u, round_up(H, 32))), 0, st,
                       pdl, 1u, hid, (const float *)nullptr, w, H, eps, 1.0f, y, ctrl, 1);
    }, "final_norm", c.block_count, (uint64_t)H * 4});
  }
  if (logits) {
    MvPlan lg = plan_matvec<Mode::PLAIN, Pro::COPY>(m->out, dev, sms);
    lg.p.xsrc = s->out_norm;
    lg.p.out = s->logits;
    lg.p.alpha = eff_scale(c.logit_scale);
    lg.p.ctrl = ctrl;
    prog.push_back({[=](cudaStream_t st, bool pdl) { return run_matvec(lg, st, pdl); }, "logits", c.block_count,
                    gguf_bytes(m->out.type, H) * m->out.g.rows});
  }
}

// ---- persistent decode-step kernel ------------------------------------------
using StepFn = void (*)(StepParams);
template <bool Q8>
StepFn pick_step_dpl(uint32_t head_dim) {
  switch (head_dim) {
    case 32: return decode_step_kernel<Q8, 1>;
    case 64: return decode_step_kernel<Q8, 2>;
    case 128: return decode_step_kernel<Q8, 4>;
    case 256: return decode_step_kernel<Q8, 8>;
  }
  return nullptr;
}

// Shared-memory plan and kernel choice of the step kernel (pointers are filled
// in by vg_stream_create). False when the model or the device does not fit it:
// the projections must share one weight format, the device must support
// cooperative launch, and one CTA with its plan must fit on an SM.
std::string plan_step(vg_stream *s) {
  vg_model *m = s->m;
  const BaseLmConfig &c = m->cfg;
  const char *env = getenv("VOXGEN_STEP_KERNEL");
  if (env && env[0] == '0') return "disabled by VOXGEN_STEP_KERNEL=0";
  const uint32_t type = m->layers[0].qkv.type;
  for (const Layer &L : m->layers)
    for (const DevMat *d : {&L.qkv, &L.o, &L.gateup, &L.down})
      if (d->type != type) return "the projections do not share one weight format";
  const int dev = m->ctx->device;
  int coop = 0;
  CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
  if (!coop) return "the device has no cooperative launch";
  const uint32_t D = c.head_dim, G = c.head_count / c.head_count_kv;
  StepParams &p = s->sp;
  p = StepParams{};
  const Layer &L0 = m->layers[0];
  p.g_qkv = L0.qkv.g;
  p.g_o = L0.o.g;
  p.g_gu = L0.gateup.g;
  p.g_down = L0.down.g;
  p.g_tok = m->tok.g;
  p.g_head = m->out.g;
  p.n_layers = c.block_count;
  p.H = c.embedding_length;
  if (m->residual) {
    // FSQ and fusion run as the step's first three phases
    for (const DevMat *d : {&m->fsq_in, &m->fsq_out, &m->fuse})
      if (d->type != type) return "the FSQ and fusion projections do not share the layers' weight format";
    p.pre = 3;
    p.g_fin = m->fsq_in.g;
    p.g_fout = m->fsq_out.g;
    p.g_fuse = m->fuse.g;
    p.w_fin = m->fsq_in.w;
    p.w_fout = m->fsq_out.w;
    p.w_fuse = m->fuse.w;
    p.b_fin = m->fsq_in_b;
    p.b_fout = m->fsq_out_b;
    p.b_fuse = m->fuse_b;
    p.fsq_scale = m->acoustic.fsq_scale;
  }
  p.xcols = 0;
  for (const TileGeom *g : {&p.g_qkv, &p.g_o, &p.g_gu, &p.g_down, &p.g_head, &p.g_fin, &p.g_fout, &p.g_fuse}) {
    if (g->cols % 4u) return strf("a matvec input of %u columns is not a whole number of 16-byte copies", g->cols);
    p.xcols = std::max(p.xcols, g->cols);
  }
  const uint32_t grid = (uint32_t)m->ctx->sms;
  uint32_t segb = 0, plane = 0, cpad = 0, rb = 1;
  s->step_head_apart = m->out.g.rows > 0 && m->out.type != type;
  if (s->step_head_apart) s->step_head = plan_matvec<Mode::PLAIN, Pro::COPY>(m->out, dev, (uint32_t)m->ctx->sms);
  for (const TileGeom *g : {&p.g_qkv, &p.g_o, &p.g_gu, &p.g_down, &p.g_head, &p.g_fin, &p.g_fout, &p.g_fuse}) {
    if (g == &p.g_head && s->step_head_apart) continue;
    if (g->rows == 0) continue;  // no LM head, or not a ResidualLM
    segb = std::max(segb, g->seg_bytes());
    const uint32_t cp = g->nseg() * g->seg_cols();
    cpad = std::max(cpad, cp);
    plane = std::max(plane, mv_a_plane(g->q8, cp));
    rb = std::max(rb, (g->tiles() + grid - 1) / grid);
  }
  p.slot = kStageSegs * segb;
  // positions per attention unit: a whole number of 16-row MMA tiles of K (or V) rows in a stage slot
  p.chunk = std::min<uint32_t>(64u, p.slot / (2u * D)) & ~15u;
  if (p.chunk == 0) return strf("a stage slot of %u bytes holds no 16 rows of head_dim %u", p.slot, D);
  if (c.head_count_kv > 64) return strf("%u KV heads (the step kernel keeps at most 64 merge counters)", c.head_count_kv);
  p.max_chunks = (s->max_ctx + p.chunk - 1) / p.chunk;
  p.plane = plane;
  p.a_bytes = std::max(round_up(3u * plane + cpad / 32u * 4u + 16u, 128u), step_attn_bytes(G, D, p.chunk, p.max_chunks));
  p.rb = rb;
  p.nst = 0;
  const uint32_t fixed = StepSmem(p).total;
  if (fixed + 2u * (p.slot + 16u) > kSmemMax) return strf("shared-memory plan of %u bytes does not fit", fixed);
  p.nst = std::min<uint32_t>(16u, (kSmemMax - fixed) / (p.slot + 16u));
  s->step_smem = StepSmem(p).total;
  s->step_fn = type == GGML_Q8_0 ? pick_step_dpl<true>(D) : pick_step_dpl<false>(D);
  if (!s->step_fn) return strf("head_dim %u", D);
  ensure_smem((const void *)s->step_fn, dev, s->step_smem);
  int per_sm = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, s->step_fn, kMvThreads, s->step_smem));
  if (per_sm < 1) return strf("no CTA of %u threads with %u bytes of shared memory fits on an SM", kMvThreads, s->step_smem);
  s->step_grid = grid;
  return "";
}

// token_input selects the token-table input of a BaseLM step; a ResidualLM
// stream has no token table, and the same flag selects its FSQ phases.
cudaError_t launch_step_kernel(vg_stream *s, bool token_input, bool logits) {
  StepParams p = s->sp;
  if (s->m->residual)
    p.fsq_on = token_input;
  else
    p.token_input = token_input;
  p.want_logits = logits && !s->step_head_apart;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(s->step_grid);
  cfg.blockDim = dim3(kMvThreads);
  cfg.dynamicSmemBytes = s->step_smem;
  cfg.stream = s->st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, s->step_fn, p);
  if (e == cudaSuccess && logits && s->step_head_apart) e = run_matvec(s->step_head, s->st, false);
  return e;
}

cudaGraphExec_t get_graph(vg_stream *s, bool token_input, bool logits) {
  cudaGraphExec_t &g = s->graphs[token_input][logits];  // ResidualLM: [fsq_on][0]
  if (g) return g;
  std::vector<Launch> prog;
  if (s->use_step) {
    prog.push_back({[=](cudaStream_t, bool) { return launch_step_kernel(s, token_input, logits); }, "step", 0, 0});
  } else {
    build_program(s, token_input, logits, prog);
  }
  cudaGraph_t graph = nullptr;
  CK(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
  cudaError_t e = cudaSuccess;
  for (size_t i = 0; i < prog.size() && e == cudaSuccess; ++i) e = prog[i].fn(s->st, i > 0);
  cudaError_t e2 = cudaStreamEndCapture(s->st, &graph);
  if (s->use_step && (e != cudaSuccess || e2 != cudaSuccess)) {
    // capture of the cooperative launch is not available: launch it directly
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    s->step_graph = false;
    return nullptr;
  }
  if (e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    fail(VG_ECUDA, strf("kernel launch during capture failed: %s", cudaGetErrorString(e)));
  }
  CK(e2);
  e = cudaGraphInstantiate(&g, graph, 0);
  cudaGraphDestroy(graph);
  CK(e);
  return g;
}

void check_step(vg_stream *s) {
  if (s->pos >= s->max_ctx)
    fail(VG_EFULL, strf("BaseLM KV cache is full at %u tokens; reset or increase --max-context", s->max_ctx));
  if (!s->m->rope_ok) fail(VG_EUNSUPPORTED, "MiniCPM4 BaseLM without LongRoPE factors is not enabled");
}

uint8_t *staging_slot(vg_stream *s) {
  const uint32_t i = s->pin_next;
  s->pin_next = (s->pin_next + 1) % kStagingSlots;
  int rc = host_wait(s->pin_ev[i], 10ull * 1000000000ull);
  if (rc) fail(rc, "timed out waiting for a staging buffer");
  return s->pin_in + (size_t)i * s->pin_in_stride;
}
cudaEvent_t staging_event(vg_stream *s) { return s->pin_ev[(s->pin_next + kStagingSlots - 1) % kStagingSlots]; }

void launch_step(vg_stream *s, bool token_input, bool logits) {
  if (logits && s->m->cfg.vocab_size == 0) fail(VG_EUNSUPPORTED, "this model has no LM head");
  cudaGraphExec_t g = s->step_graph ? get_graph(s, token_input, logits) : nullptr;
  if (g)
    CK(cudaGraphLaunch(g, s->st));
  else
    CK(launch_step_kernel(s, token_input, logits));
  s->pos += 1;
  s->logits_valid = logits;
}

// One ResidualLM position on the step kernel (FSQ phases on or off).
void launch_residual_step(vg_stream *s, bool fsq) {
  cudaGraphExec_t g = s->step_graph ? get_graph(s, fsq, false) : nullptr;
  if (g)
    CK(cudaGraphLaunch(g, s->st));
  else
    CK(launch_step_kernel(s, fsq, false));
  s->pos += 1;
  s->logits_valid = false;
}

int sync_stream(vg_stream *s, uint64_t timeout_ns, bool check_flag) {
  CK(cudaEventRecord(s->ev_done, s->st));
  int rc = host_wait(s->ev_done, timeout_ns);
  if (rc) fail(rc, "stream did not finish within the timeout");
  if (check_flag) {
    uint32_t flag = 0;
    CK(cudaMemcpy(&flag, s->ctrl + kCtrlErr, 4, cudaMemcpyDeviceToHost));
    if (flag) {
      CK(cudaMemset(s->ctrl + kCtrlErr, 0, 4));
      fail(VG_EDEVICE, strf("a kernel raised device error flag 0x%x", flag));
    }
  }
  return VG_OK;
}

void destroy_stream(vg_stream *s) {
  for (auto &row : s->graphs)
    for (auto &g : row)
      if (g) cudaGraphExecDestroy(g);
  for (auto &e : s->pin_ev)
    if (e) cudaEventDestroy(e);
  if (s->ev_done) cudaEventDestroy(s->ev_done);
  if (s->st) cudaStreamDestroy(s->st);
  if (s->kc) cudaFree(s->kc);
  if (s->dev_block) cudaFree(s->dev_block);
  if (s->pin_in) cudaFreeHost(s->pin_in);
  if (s->pin_out) cudaFreeHost(s->pin_out);
}

// ---- batched step kernel ---------------------------------------------------
using BatchFn = void (*)(BatchParams);
template <bool Q8>
BatchFn pick_batch_dpl(uint32_t head_dim) {
  switch (head_dim) {
    case 32: return decode_batch_kernel<Q8, 1>;
    case 64: return decode_batch_kernel<Q8, 2>;
    case 128: return decode_batch_kernel<Q8, 4>;
  }
  // a warp's attention unit at head_dim 256 would spill its output tile; such
  // models step each stream with its own launch
  return nullptr;
}

// Column groups of one matvec kind: the split with the smallest estimate of
// the phase time, the heaviest CTA's weight bytes at its share of HBM
// bandwidth plus the L2 traffic of operand slices (one read per row group)
// and partial sums (written and read once per column group). A CTA's slice
// must fit the operand region and span at most 8 segments.
BatchSplit choose_split(const TileGeom &g, uint32_t S, uint32_t grid, uint32_t max_aux) {
  const double sm_bw = 6.5e12 / grid, l2_bw = 10e12;  // B/s: HBM share of one SM; L2 (estimate)
  BatchSplit best{0, 0};
  double bc = 1e300;
  for (uint32_t C = 1; C <= std::min(g.nseg(), grid); ++C) {
    const uint32_t R = grid / C;
    const uint32_t ns = (g.nseg() + C - 1) / C, nt = (g.tiles() + R - 1) / R;
    if (ns > 8 || BatchOperand(ns * g.seg_cols()).total > max_aux) continue;
    const double hbm = (double)nt * ns * g.seg_bytes() / sm_bw;
    const double l2 = ((double)R * S * g.cols * 4.0 + (double)C * g.tiles() * 256.0 * 4.0 * 2.0) / l2_bw;
    if (hbm + l2 < bc) {
      bc = hbm + l2;
      best = {C, R};
    }
  }
  return best;
}

void destroy_batch(vg_model *m) {
  BatchWork *w = m->batch;
  if (!w) return;
  if (w->st) cudaStreamSynchronize(w->st);
  for (auto &e : w->pin_ev)
    if (e) cudaEventDestroy(e);
  if (w->ev_done) cudaEventDestroy(w->ev_done);
  if (w->st) cudaStreamDestroy(w->st);
  if (w->dev) cudaFree(w->dev);
  if (w->pin) cudaFreeHost(w->pin);
  delete w;
  m->batch = nullptr;
}

// Plans the batched kernel for model m into w; returns "" or why it cannot run.
std::string plan_batch(vg_model *m, BatchWork &w) {
  const char *env = getenv("VOXGEN_BATCH_KERNEL");
  if (env && env[0] == '0') return "disabled by VOXGEN_BATCH_KERNEL=0";
  if (m->residual) return "a ResidualLM model";
  const BaseLmConfig &c = m->cfg;
  const uint32_t type = m->layers[0].qkv.type;
  for (const Layer &L : m->layers)
    for (const DevMat *d : {&L.qkv, &L.o, &L.gateup, &L.down})
      if (d->type != type) return "the projections do not share one weight format";
  const int dev = m->ctx->device;
  int coop = 0;
  CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
  if (!coop) return "the device has no cooperative launch";
  const uint32_t D = c.head_dim, G = c.head_count / c.head_count_kv, H = c.embedding_length;
  if (c.head_count_kv > 8) return strf("%u KV heads (at most 8)", c.head_count_kv);
  if (G > 8 || G % 2) return strf("%u query heads per KV head (an even count up to 8)", G);
  if (c.head_count * D != H) return "the query width differs from the hidden width";
  w.fn = type == GGML_Q8_0 ? pick_batch_dpl<true>(D) : pick_batch_dpl<false>(D);
  if (!w.fn) return strf("head_dim %u (the batched kernel takes 32, 64 or 128)", D);
  BatchParams &p = w.p;
  p = BatchParams{};
  const Layer &L0 = m->layers[0];
  p.g[kBkQkv] = L0.qkv.g;
  p.g[kBkO] = L0.o.g;
  p.g[kBkGu] = L0.gateup.g;
  p.g[kBkDown] = L0.down.g;
  p.g_tok = m->tok.g;
  p.n_layers = c.block_count;
  uint32_t segb = 0, part_tiles = 0;
  for (const TileGeom &g : p.g) {
    if (g.cols % 4u) return strf("a matvec input of %u columns is not a whole number of 16-byte copies", g.cols);
    segb = std::max(segb, g.seg_bytes());
    part_tiles = std::max(part_tiles, g.tiles());
  }
  p.slot = kStageSegs * segb;
  // positions per attention unit: 16-row MMA tiles of K and V rows, both in one stage slot
  p.chunk = batch_chunk(D);
  if (4u * p.chunk * D > p.slot) return strf("a stage slot of %u bytes holds no %u K and V rows of head_dim %u", p.slot, p.chunk, D);
  p.max_chunks = (c.context_length + p.chunk - 1) / p.chunk;
  const uint32_t grid = (uint32_t)m->ctx->sms;
  if (grid > kBatchMaxRowGroups) return strf("%u SMs (the row-group counters cover %u)", grid, kBatchMaxRowGroups);
  constexpr uint32_t kMaxAux = 72u * 1024u;  // operand region: leaves the ring 8 or more stages
  uint32_t aux = batch_attn_bytes(p.chunk, p.max_chunks), maxc = 1;
  for (uint32_t k = 0; k < kBatchKinds; ++k) {
    const TileGeom &g = p.g[k];
    p.split[k] = choose_split(g, kBatchMaxCols, grid, kMaxAux);
    if (p.split[k].C == 0) return strf("no split of a %u x %u matrix fits the operand region", g.rows, g.cols);
    const uint32_t ns = (g.nseg() + p.split[k].C - 1) / p.split[k].C;
    aux = std::max(aux, BatchOperand(ns * g.seg_cols()).total);
    maxc = std::max(maxc, p.split[k].C);
  }
  p.aux_bytes = aux;
  p.nst = 0;
  const uint32_t fixed = BatchSmem(p).total;
  if (fixed + 4u * (p.slot + 16u) > kSmemMax) return strf("shared-memory plan of %u bytes does not fit", fixed);
  p.nst = std::min<uint32_t>(16u, (kSmemMax - fixed) / (p.slot + 16u));
  w.smem = BatchSmem(p).total;
  ensure_smem((const void *)w.fn, dev, w.smem);
  int per_sm = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, w.fn, kMvThreads, w.smem));
  if (per_sm < 1) return strf("no CTA with %u bytes of shared memory fits on an SM", w.smem);
  w.grid = grid;
  // workspace
  const uint32_t S = kBatchMaxCols, F = c.feed_forward_length, KVH = c.head_count_kv;
  size_t off = 0;
  auto take = [&](size_t b) {
    size_t o = off;
    off = round_up_sz(off + b, 256);
    return o;
  };
  w.table_bytes = S * sizeof(BatchCol) + kCtrlWords * 4;
  const size_t o_cols = take(w.table_bytes);
  const size_t o_a = take((size_t)S * H * 4), o_b = take((size_t)S * H * 4), o_q = take((size_t)S * H * 4),
               o_at = take((size_t)S * H * 4), o_g = take((size_t)S * F * 4),
               o_part = take((size_t)maxc * part_tiles * 256 * 4), o_ssb = take((size_t)grid * S * 4),
               o_ap = take((size_t)S * KVH * p.max_chunks * G * D * 4),
               o_ml = take((size_t)S * KVH * p.max_chunks * G * 8), o_rdy = take((size_t)S * KVH * 8),
               o_rgc = take((size_t)kBatchKinds * kBatchMaxRowGroups * 8), o_bar = take(8),
               o_ly = take((size_t)c.block_count * sizeof(StepLayer));
  CK(cudaMalloc(&w.dev, off));
  CK(cudaMemset(w.dev, 0, off));
  uint8_t *b = static_cast<uint8_t *>(w.dev);
  p.cols = reinterpret_cast<const BatchCol *>(b + o_cols);
  p.ctrl = reinterpret_cast<uint32_t *>(b + o_cols + S * sizeof(BatchCol));
  p.hid_a = (float *)(b + o_a);
  p.hid_b = (float *)(b + o_b);
  p.q = (float *)(b + o_q);
  p.attn = (float *)(b + o_at);
  p.gate = (float *)(b + o_g);
  p.part = (float *)(b + o_part);
  p.part_tiles = part_tiles;
  p.ssb = (float *)(b + o_ssb);
  p.apart = (float *)(b + o_ap);
  p.apart_ml = (float2 *)(b + o_ml);
  p.ready = (unsigned long long *)(b + o_rdy);
  p.rgc = (unsigned long long *)(b + o_rgc);
  p.bar = (unsigned long long *)(b + o_bar);
  std::vector<StepLayer> tab(c.block_count);
  for (uint32_t l = 0; l < c.block_count; ++l) {
    const Layer &L = m->layers[l];
    tab[l] = StepLayer{L.qkv.w, L.o.w, L.gateup.w, L.down.w, L.attn_norm, L.ffn_norm, nullptr, nullptr};
  }
  CK(cudaMemcpy(b + o_ly, tab.data(), tab.size() * sizeof(StepLayer), cudaMemcpyHostToDevice));
  p.layers = (const StepLayer *)(b + o_ly);
  p.tok = m->tok.w;
  p.out_norm = m->out_norm;
  p.inv_freq = m->inv_freq;
  p.ext = m->ext;
  p.rope_scaling = c.rope_scaling_factor();
  p.eps = c.rms_epsilon;
  p.res_scale = eff_scale(c.residual_scale);
  p.emb_scale = eff_scale(c.embedding_scale);
  p.attn_scale = 1.0f / sqrtf((float)D);
  p.H = H;
  p.F = F;
  p.heads = c.head_count;
  p.kv_heads = KVH;
  p.head_dim = D;
  CK(cudaStreamCreateWithFlags(&w.st, cudaStreamNonBlocking));
  CK(cudaEventCreateWithFlags(&w.ev_done, cudaEventDisableTiming));
  w.pin_stride = round_up_sz(w.table_bytes, 256);
  CK(cudaMallocHost(&w.pin, w.pin_stride * kBatchStaging));
  for (auto &e : w.pin_ev) {
    CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    CK(cudaEventRecord(e, w.st));
  }
  CK(cudaStreamSynchronize(w.st));
  return "";
}

// The model's batch plan, made at first use (caller holds m->batch_mu).
BatchWork *get_batch(vg_model *m) {
  if (!m->batch) {
    m->batch = new BatchWork();
    try {
      m->batch->why = plan_batch(m, *m->batch);
    } catch (...) {
      destroy_batch(m);
      throw;
    }
  }
  return m->batch;
}

BatchCol batch_col(const vg_stream *s, uint32_t off, uint32_t adv, uint32_t token) {
  const BaseLmConfig &c = s->m->cfg;
  BatchCol col{};
  col.kc = s->kc;
  col.vc = s->vc;
  col.layer_elems = (unsigned long long)c.head_count_kv * s->max_ctx * c.head_dim;
  col.ctrl = s->ctrl;
  col.out = s->out_norm;
  col.ctx = s->max_ctx;
  col.off = off;
  col.adv = adv;
  col.token = token;
  return col;
}

// One launch of the batched kernel over cols (caller holds m->batch_mu),
// ordered after the work already enqueued on every stream involved and
// before their later work. The column table and a clean control block travel
// with the launch.
void batch_launch(BatchWork &w, const std::vector<BatchCol> &cols, const std::vector<vg_stream *> &streams) {
  const uint32_t i = w.pin_next;
  w.pin_next = (w.pin_next + 1) % kBatchStaging;
  int rc = host_wait(w.pin_ev[i], 10ull * 1000000000ull);
  if (rc) fail(rc, "timed out waiting for a batch staging buffer");
  uint8_t *slot = w.pin + (size_t)i * w.pin_stride;
  std::memset(slot, 0, w.table_bytes);
  std::memcpy(slot, cols.data(), cols.size() * sizeof(BatchCol));
  for (vg_stream *s : streams) {
    CK(cudaEventRecord(s->ev_done, s->st));
    CK(cudaStreamWaitEvent(w.st, s->ev_done, 0));
  }
  CK(cudaMemcpyAsync((void *)w.p.cols, slot, w.table_bytes, cudaMemcpyHostToDevice, w.st));
  CK(cudaEventRecord(w.pin_ev[i], w.st));
  BatchParams p = w.p;
  p.S = (uint32_t)cols.size();
  p.merge_dw = batch_merge_width(p.S, p.kv_heads, p.head_dim, p.heads / p.kv_heads, w.grid);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(w.grid);
  cfg.blockDim = dim3(kMvThreads);
  cfg.dynamicSmemBytes = w.smem;
  cfg.stream = w.st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  CK(cudaLaunchKernelEx(&cfg, w.fn, p));
  CK(cudaEventRecord(w.ev_done, w.st));
  for (vg_stream *s : streams) CK(cudaStreamWaitEvent(s->st, w.ev_done, 0));
}

}  // namespace

// ===========================================================================
// ABI
// ===========================================================================
extern "C" {

int vg_ctx_create(int device, vg_ctx **out) {
  if (!out) return VG_EINVAL;
  *out = nullptr;
  vg_ctx *c = new vg_ctx();
  c->device = device;
  int rc = guard(c, [&] {
    int n = 0;
    CK(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) fail(VG_EINVAL, strf("device %d out of range (%d devices)", device, n));
    CK(cudaSetDevice(device));
    CK(cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, device));
    return VG_OK;
  });
  if (rc) {
    delete c;
    return rc;
  }
  live_add(c);
  *out = c;
  return VG_OK;
}

int vg_ctx_destroy(vg_ctx *c) {
  if (!live(c)) return VG_ESTATE;
  live_del(c);
  delete c;
  return VG_OK;
}

const char *vg_last_error(const vg_ctx *c) {
  if (!live(c)) return "invalid or destroyed context";
  return c->err.c_str();
}

int vg_ctx_sm_count(const vg_ctx *c, int *out) {
  if (!live(c) || !out) return live(c) ? VG_EINVAL : VG_ESTATE;
  *out = c->sms;
  return VG_OK;
}

int vg_gguf_inspect(const char *path, int format, vg_model_info *info, char *err, size_t err_len) {
  if (err && err_len) err[0] = 0;
  if (!path || !info) return VG_EINVAL;
  if (format != VG_FORMAT_AUTO && format != VG_FORMAT_Q8_0 && format != VG_FORMAT_F16) return VG_EINVAL;
  try {
    vg_model tmp;
    tmp.summary = load_summary(path);
    tmp.cfg = config_from_gguf(tmp.summary, (uint32_t)format);
    check_kernel_support(tmp.summary, tmp.cfg);
    // device bytes the repack would take (same layout as load_model)
    const BaseLmConfig &c = tmp.cfg;
    size_t bytes = 0;
    auto add = [&](size_t b) { bytes = round_up_sz(bytes + b, 256); };
    for (uint32_t l = 0; l < c.block_count; ++l) {
      auto t = [&](const char *s) { return tmp.summary.find(strf("blk.%u.%s.weight", l, s))->type; };
      add(packed_bytes(t("attn_q"), c.embedding_length + 2 * c.kv_dim, c.embedding_length));
      add(packed_bytes(t("attn_output"), c.embedding_length, c.embedding_length));
      add(packed_bytes(t("ffn_gate"), 2 * c.feed_forward_length, c.embedding_length));
      add(packed_bytes(t("ffn_down"), c.embedding_length, c.feed_forward_length));
      add((size_t)c.embedding_length * 4);
      add((size_t)c.embedding_length * 4);
    }
    add(packed_bytes(tmp.summary.find("token_embd.weight")->type, c.vocab_size, c.embedding_length));
    if (!c.tied_output)
      add(packed_bytes(tmp.summary.find("output.weight")->type, c.vocab_size, c.embedding_length));
    add((size_t)c.embedding_length * 4);
    add((size_t)c.head_dim / 2 * 4);
    add((size_t)c.head_dim / 2 * 4);
    tmp.arena_bytes = bytes;
    fill_info(&tmp);
    *info = tmp.info;
    return VG_OK;
  } catch (const Error &e) {
    if (err && err_len) snprintf(err, err_len, "%s", e.msg.c_str());
    return e.code;
  } catch (const std::exception &e) {
    if (err && err_len) snprintf(err, err_len, "%s", e.what());
    return VG_EINVAL;
  }
}

int vg_kv_cache_bytes(const vg_model_info *info, uint32_t max_context, uint64_t *bytes) {
  if (!info || !bytes) return VG_EINVAL;
  *bytes = (uint64_t)info->block_count * max_context * info->kv_dim * 2 /* fp16 */ * 2 /* K + V */;
  return VG_OK;
}

int vg_top_k_logits(const float *logits, uint32_t n, uint32_t k, vg_top_logit *out, uint32_t *n_out) {
  if ((!logits && n) || (!out && k) || !n_out) return VG_EINVAL;
  // finite values only, descending; equal values keep index order
  std::vector<uint32_t> idx;
  idx.reserve(n);
  for (uint32_t i = 0; i < n; ++i)
    if (std::isfinite(logits[i])) idx.push_back(i);
  const size_t kk = std::min<size_t>(k, idx.size());
  std::partial_sort(idx.begin(), idx.begin() + kk, idx.end(), [&](uint32_t a, uint32_t b) {
    return logits[a] > logits[b] || (logits[a] == logits[b] && a < b);
  });
  for (size_t i = 0; i < kk; ++i) out[i] = {idx[i], logits[idx[i]]};
  *n_out = (uint32_t)kk;
  return VG_OK;
}

int vg_model_load_gguf(vg_ctx *ctx, const char *path, int format, vg_model **out) {
  if (!live(ctx)) return VG_ESTATE;
  if (!path || !out) return VG_EINVAL;
  *out = nullptr;
  if (format != VG_FORMAT_AUTO && format != VG_FORMAT_Q8_0 && format != VG_FORMAT_F16) return VG_EINVAL;
  vg_model *m = new vg_model();
  m->ctx = ctx;
  int rc = guard(ctx, [&] {
    CK(cudaSetDevice(ctx->device));
    load_model(m, path, (uint32_t)format);
    return VG_OK;
  });
  if (rc) {
    if (m->arena) cudaFree(m->arena);
    delete m;
    return rc;
  }
  live_add(m);
  *out = m;
  return VG_OK;
}

int vg_model_info_get(const vg_model *m, vg_model_info *info) {
  if (!live(m)) return VG_ESTATE;
  if (!info) return VG_EINVAL;
  *info = m->info;
  return VG_OK;
}

int vg_model_destroy(vg_model *m) {
  if (!live(m)) return VG_ESTATE;
  if (m->streams > 0) {
    set_err(m->ctx, "model still has live streams");
    return VG_ESTATE;
  }
  live_del(m);
  cudaSetDevice(m->ctx->device);
  destroy_batch(m);
  if (m->arena) cudaFree(m->arena);
  delete m;
  return VG_OK;
}

int vg_stream_create(vg_model *m, uint32_t max_context, vg_stream **out) {
  if (!live(m)) return VG_ESTATE;
  if (!out) return VG_EINVAL;
  *out = nullptr;
  vg_stream *s = new vg_stream();
  s->m = m;
  int rc = guard(m->ctx, [&] {
    const BaseLmConfig &c = m->cfg;
    // BaseLmConfig::from_gguf, src/baselm.rs:68-72
    if (max_context == 0 || max_context > c.context_length)
      fail(VG_EINVAL, strf("--max-context must be in 1..=%u, got %u", c.context_length, max_context));
    CK(cudaSetDevice(m->ctx->device));
    s->max_ctx = max_context;
    const uint32_t H = c.embedding_length, D = c.head_dim, G = c.head_count / c.head_count_kv;
    plan_attention(max_context, s->nsplit, s->chunk_cap);
    const std::string why = plan_step(s);
    s->use_step = why.empty();
    const char *want = getenv("VOXGEN_STEP_KERNEL");
    if (!s->use_step && want && want[0] == '1')
      fail(VG_EUNSUPPORTED, "persistent step kernel required by VOXGEN_STEP_KERNEL=1 but unavailable: " + why);
    const uint32_t nch = s->use_step ? s->sp.max_chunks : 0u;
    const size_t kv_elems = (size_t)c.block_count * c.head_count_kv * max_context * D;
    CK(cudaMalloc(&s->kc, kv_elems * 2 * sizeof(__half)));
    s->vc = s->kc + kv_elems;
    // activations + scratch + control, one allocation
    size_t off = 0;
    auto take = [&](size_t b) {
      size_t o = off;
      off = round_up_sz(off + b, 256);
      return o;
    };
    const size_t o_out = take((size_t)H * 4), o_ctrl = take(kCtrlWords * 4);
    const size_t o_a = take((size_t)H * 4), o_b = take((size_t)H * 4), o_q = take((size_t)H * 4),
                 o_att = take((size_t)H * 4), o_g = take((size_t)c.feed_forward_length * 4),
                 o_lg = take((size_t)c.vocab_size * 4),
                 o_part = take((size_t)c.head_count_kv * (s->nsplit / kAttnCluster) * G * (D + 2) * 4),
                 o_tk = take((size_t)c.head_count_kv * G * 4),
                 o_bar = take(8), o_sl = take((size_t)c.block_count * sizeof(StepLayer)),
                 o_sp = take((size_t)c.head_count_kv * nch * G * D * 4),
                 o_sml = take((size_t)c.head_count_kv * nch * G * 8),
                 o_rdy = take((size_t)c.head_count_kv * 8);
    const uint32_t LAT = m->residual ? m->acoustic.fsq_latent_dim : 0u, HR = m->residual ? H : 0u;
    const size_t o_rb = take((size_t)HR * 4), o_rl = take((size_t)LAT * 4), o_rf = take((size_t)HR * 4),
                 o_ri = take((size_t)HR * 8), o_rs = take((size_t)HR * 4);
    CK(cudaMalloc(&s->dev_block, off));
    CK(cudaMemset(s->dev_block, 0, off));
    uint8_t *b = static_cast<uint8_t *>(s->dev_block);
    s->out_norm = (float *)(b + o_out);
    s->ctrl = (uint32_t *)(b + o_ctrl);
    s->hid_a = (float *)(b + o_a);
    s->hid_b = (float *)(b + o_b);
    s->q = (float *)(b + o_q);
    s->attn = (float *)(b + o_att);
    s->gate = (float *)(b + o_g);
    s->logits = (float *)(b + o_lg);
    s->part = (float *)(b + o_part);
    s->tickets = (uint32_t *)(b + o_tk);
    if (m->residual) {
      s->res_base = (float *)(b + o_rb);
      s->fsq_lat = (float *)(b + o_rl);
      s->fsq_res = (float *)(b + o_rf);
      s->fuse_in = (float *)(b + o_ri);
      s->fused = (float *)(b + o_rs);
      const int dev = m->ctx->device;
      const uint32_t sms = (uint32_t)m->ctx->sms;
      // linear_bias.comp / fusion_linear.comp: (W x + bias), the bias as the residual
      auto plan = [&](const DevMat &w, const float *x, float *y, const float *bias) {
        MvPlan pl = plan_matvec<Mode::RESID, Pro::COPY>(w, dev, sms);
        pl.p.xsrc = x;
        pl.p.out = y;
        pl.p.resid = bias;
        pl.p.alpha = 1.0f;
        pl.p.ctrl = s->ctrl;
        return pl;
      };
      s->fsq_in_p = plan(m->fsq_in, s->res_base, s->fsq_lat, m->fsq_in_b);
      s->fsq_out_p = plan(m->fsq_out, s->fsq_lat, s->fsq_res, m->fsq_out_b);
      s->fuse_p = plan(m->fuse, s->fuse_in, s->fused, m->fuse_b);
    }
    if (s->use_step) {
      StepParams &p = s->sp;
      std::vector<StepLayer> tab(c.block_count);
      const size_t per_layer = (size_t)c.head_count_kv * max_context * D;
      for (uint32_t l = 0; l < c.block_count; ++l) {
        const Layer &L = m->layers[l];
        tab[l] = StepLayer{L.qkv.w, L.o.w, L.gateup.w, L.down.w, L.attn_norm, L.ffn_norm,
                           s->kc + l * per_layer, s->vc + l * per_layer};
      }
      CK(cudaMemcpy(b + o_sl, tab.data(), tab.size() * sizeof(StepLayer), cudaMemcpyHostToDevice));
      p.layers = (const StepLayer *)(b + o_sl);
      p.tok = m->tok.w;
      p.head = m->out.w;
      p.out_norm = m->out_norm;
      p.hid_a = s->hid_a;
      p.hid_b = s->hid_b;
      p.q = s->q;
      p.attn = s->attn;
      p.gate = s->gate;
      p.logits = s->logits;
      p.out = s->out_norm;
      if (s->step_head_apart) {
        MvParams &hp = s->step_head.p;
        hp.xsrc = s->out_norm;
        hp.out = s->logits;
        hp.alpha = eff_scale(c.logit_scale);
        hp.ctrl = s->ctrl;
      }
      p.part = (float *)(b + o_sp);
      p.part_ml = (float2 *)(b + o_sml);
      p.ready = (unsigned long long *)(b + o_rdy);
      if (m->residual) {
        p.res_base = s->res_base;
        p.fsq_lat = s->fsq_lat;
        p.fsq_res = s->fsq_res;
        p.fuse_in = s->fuse_in;
        p.fused = s->fused;
      }
      p.inv_freq = m->inv_freq;
      p.ext = m->ext;
      p.rope_scaling = c.rope_scaling_factor();
      p.eps = c.rms_epsilon;
      p.res_scale = eff_scale(c.residual_scale);
      p.emb_scale = eff_scale(c.embedding_scale);
      p.logit_scale = eff_scale(c.logit_scale);
      p.attn_scale = 1.0f / sqrtf((float)D);
      p.H = H;
      p.F = c.feed_forward_length;
      p.heads = c.head_count;
      p.kv_heads = c.head_count_kv;
      p.head_dim = D;
      p.ctx = max_context;
      p.ctrl = s->ctrl;
      p.bar = (unsigned long long *)(b + o_bar);
    }
    CK(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&s->ev_done, cudaEventDisableTiming));
    s->pin_in_stride = round_up_sz(16 + (size_t)H * 4, 256);
    CK(cudaMallocHost(&s->pin_in, s->pin_in_stride * kStagingSlots));
    for (auto &e : s->pin_ev) {
      CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      CK(cudaEventRecord(e, s->st));
    }
    CK(cudaMallocHost(&s->pin_out, round_up_sz((size_t)std::max(H, c.vocab_size) * 4, 256) + 256));
    CK(cudaStreamSynchronize(s->st));
    return VG_OK;
  });
  if (rc) {
    destroy_stream(s);
    delete s;
    return rc;
  }
  m->streams += 1;
  live_add(s);
  *out = s;
  return VG_OK;
}

int vg_stream_destroy(vg_stream *s) {
  if (!live(s)) return VG_ESTATE;
  live_del(s);
  cudaSetDevice(s->m->ctx->device);
  cudaStreamSynchronize(s->st);
  s->m->streams -= 1;
  destroy_stream(s);
  delete s;
  return VG_OK;
}

int vg_stream_reset(vg_stream *s) {
  if (!live(s)) return VG_ESTATE;
  return guard(s->m->ctx, [&] {
    CK(cudaSetDevice(s->m->ctx->device));
    // Cache contents stay; they are unreachable once the position is 0 (src/baselm.rs:616-620).
    CK(cudaMemsetAsync(s->ctrl + kCtrlPos, 0, 4, s->st));
    s->pos = 0;
    return VG_OK;
  });
}

int vg_stream_position(const vg_stream *s, uint32_t *position) {
  if (!live(s)) return VG_ESTATE;
  if (!position) return VG_EINVAL;
  *position = s->pos;
  return VG_OK;
}

int vg_stream_seek(vg_stream *s, uint32_t position) {
  if (!live(s)) return VG_ESTATE;
  return guard(s->m->ctx, [&] {
    if (position > s->max_ctx) fail(VG_EINVAL, strf("position %u is beyond the KV cache of %u", position, s->max_ctx));
    CK(cudaSetDevice(s->m->ctx->device));
    uint8_t *slot = staging_slot(s);
    std::memcpy(slot, &position, 4);
    CK(cudaMemcpyAsync(s->ctrl + kCtrlPos, slot, 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaEventRecord(staging_event(s), s->st));
    s->pos = position;
    return VG_OK;
  });
}

int vg_stream_set_wait_limit(vg_stream *s, uint64_t limit_ns) {
  if (!live(s)) return VG_ESTATE;
  if (limit_ns > 0xFFFFFFFFull) {
    set_err(s->m->ctx, "device wait limit above 4294967295 ns");
    return VG_EINVAL;
  }
  return guard(s->m->ctx, [&] {
    CK(cudaSetDevice(s->m->ctx->device));
    const uint32_t v = (uint32_t)limit_ns;
    uint8_t *slot = staging_slot(s);
    std::memcpy(slot, &v, 4);
    CK(cudaMemcpyAsync(s->ctrl + kCtrlWaitNs, slot, 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaEventRecord(staging_event(s), s->st));
    return VG_OK;
  });
}

int vg_test_stalled_step(vg_stream *s, uint32_t token) {
  if (!live(s)) return VG_ESTATE;
  return guard(s->m->ctx, [&] {
    if (!s->use_step) fail(VG_EUNSUPPORTED, "the stalled-barrier test needs the persistent step kernel");
    if (token >= s->m->cfg.vocab_size)
      fail(VG_ERANGE, strf("token id %u is outside vocabulary 0..%u", token, s->m->cfg.vocab_size));
    check_step(s);
    CK(cudaSetDevice(s->m->ctx->device));
    uint8_t *slot = staging_slot(s);
    const uint32_t words[3] = {token, 1u, 0u};  // token, one missing barrier arrival, then its reset
    std::memcpy(slot, words, sizeof words);
    CK(cudaMemcpyAsync(s->ctrl + kCtrlToken, slot, 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaMemcpyAsync(s->ctrl + kCtrlBarExtra, slot + 4, 4, cudaMemcpyHostToDevice, s->st));
    launch_step(s, true, false);
    CK(cudaMemcpyAsync(s->ctrl + kCtrlBarExtra, slot + 8, 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaEventRecord(staging_event(s), s->st));
    return VG_OK;
  });
}

int vg_test_fake_event_status(int status) {
  g_fake_event_status.store(status, std::memory_order_relaxed);
  return VG_OK;
}

int vg_stream_kernel_mode(const vg_stream *s, int *mode) {
  if (!live(s)) return VG_ESTATE;
  if (!mode) return VG_EINVAL;
  *mode = s->use_step ? 1 : 0;
  return VG_OK;
}

int vg_stream_cuda_stream(const vg_stream *s, void **cuda_stream) {
  if (!live(s)) return VG_ESTATE;
  if (!cuda_stream) return VG_EINVAL;
  *cuda_stream = (void *)s->st;
  return VG_OK;
}

int vg_stream_write_kv(vg_stream *s, const uint16_t *k, const uint16_t *v, uint32_t n) {
  if (!live(s)) return VG_ESTATE;
  if ((!k || !v) && n) return VG_EINVAL;
  return guard(s->m->ctx, [&] {
    const BaseLmConfig &c = s->m->cfg;
    if (n > s->max_ctx) fail(VG_EFULL, strf("%u positions exceed the KV cache of %u", n, s->max_ctx));
    CK(cudaSetDevice(s->m->ctx->device));
    CK(cudaStreamSynchronize(s->st));
    // reference layout [layer][pos][kv_dim] -> [layer][kv_head][ctx][head_dim],
    // each row's chunks permuted as kv_swz stores them
    const uint32_t D = c.head_dim;
    std::vector<uint16_t> blk((size_t)n * D);
    for (uint32_t l = 0; l < c.block_count && n; ++l)
      for (uint32_t h = 0; h < c.head_count_kv; ++h) {
        const size_t dst = ((size_t)l * c.head_count_kv + h) * s->max_ctx * D;
        for (int which = 0; which < 2; ++which) {
          const uint16_t *src = (which ? v : k) + (size_t)l * n * c.kv_dim + (size_t)h * D;
          for (uint32_t pos = 0; pos < n; ++pos)
            for (uint32_t e = 0; e < D; ++e) blk[(size_t)pos * D + kv_swz(pos, e, D)] = src[(size_t)pos * c.kv_dim + e];
          CK(cudaMemcpy((which ? s->vc : s->kc) + dst, blk.data(), blk.size() * 2, cudaMemcpyHostToDevice));
        }
      }
    CK(cudaMemcpy(s->ctrl + kCtrlPos, &n, 4, cudaMemcpyHostToDevice));
    s->pos = n;
    return VG_OK;
  });
}

int vg_stream_read_kv(vg_stream *s, uint16_t *k, uint16_t *v, uint32_t n) {
  if (!live(s)) return VG_ESTATE;
  if ((!k || !v) && n) return VG_EINVAL;
  return guard(s->m->ctx, [&] {
    const BaseLmConfig &c = s->m->cfg;
    if (n > s->max_ctx) fail(VG_EINVAL, strf("%u positions exceed the KV cache of %u", n, s->max_ctx));
    CK(cudaSetDevice(s->m->ctx->device));
    sync_stream(s, 60ull * 1000000000ull, false);
    const uint32_t D = c.head_dim;
    std::vector<uint16_t> blk((size_t)n * D);
    for (uint32_t l = 0; l < c.block_count && n; ++l)
      for (uint32_t h = 0; h < c.head_count_kv; ++h) {
        const size_t src = ((size_t)l * c.head_count_kv + h) * s->max_ctx * D;
        for (int which = 0; which < 2; ++which) {
          CK(cudaMemcpy(blk.data(), (which ? s->vc : s->kc) + src, blk.size() * 2, cudaMemcpyDeviceToHost));
          uint16_t *dst = (which ? v : k) + (size_t)l * n * c.kv_dim + (size_t)h * D;
          for (uint32_t pos = 0; pos < n; ++pos)
            for (uint32_t e = 0; e < D; ++e) dst[(size_t)pos * c.kv_dim + e] = blk[(size_t)pos * D + kv_swz(pos, e, D)];
        }
      }
    return VG_OK;
  });
}

int vg_decode_token(vg_stream *s, uint32_t token, int want_logits) {
  if (!live(s)) return VG_ESTATE;
  return guard(s->m->ctx, [&] {
    if (token >= s->m->cfg.vocab_size)
      fail(VG_ERANGE, strf("token id %u is outside vocabulary 0..%u", token, s->m->cfg.vocab_size));
    check_step(s);
    CK(cudaSetDevice(s->m->ctx->device));
    uint8_t *slot = staging_slot(s);
    std::memcpy(slot, &token, 4);
    CK(cudaMemcpyAsync(s->ctrl + kCtrlToken, slot, 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaEventRecord(staging_event(s), s->st));
    launch_step(s, true, want_logits != 0);
    return VG_OK;
  });
}

int vg_decode_embedding(vg_stream *s, const float *host, int want_logits) {
  if (!live(s)) return VG_ESTATE;
  if (!host) return VG_EINVAL;
  return guard(s->m->ctx, [&] {
    check_step(s);
    CK(cudaSetDevice(s->m->ctx->device));
    const size_t bytes = (size_t)s->m->cfg.embedding_length * 4;
    uint8_t *slot = staging_slot(s);
    std::memcpy(slot + 16, host, bytes);
    CK(cudaMemcpyAsync(s->hid_a, slot + 16, bytes, cudaMemcpyHostToDevice, s->st));
    CK(cudaEventRecord(staging_event(s), s->st));
    launch_step(s, false, want_logits != 0);
    return VG_OK;
  });
}

int vg_decode_embedding_device(vg_stream *s, const float *dev, int want_logits) {
  if (!live(s)) return VG_ESTATE;
  if (!dev) return VG_EINVAL;
  return guard(s->m->ctx, [&] {
    check_step(s);
    CK(cudaSetDevice(s->m->ctx->device));
    CK(cudaMemcpyAsync(s->hid_a, dev, (size_t)s->m->cfg.embedding_length * 4, cudaMemcpyDeviceToDevice, s->st));
    launch_step(s, false, want_logits != 0);
    return VG_OK;
  });
}

// ---- ResidualLM + FSQ + fusion (acoustic GGUF) -------------------------------

int vg_residual_load_gguf(vg_ctx *ctx, const char *path, const vg_model *base, vg_model **out) {
  if (!live(ctx) || !live(base)) return VG_ESTATE;
  if (!path || !out) return VG_EINVAL;
  *out = nullptr;
  if (base->residual || base->ctx != ctx) return VG_EINVAL;
  vg_model *m = new vg_model();
  m->ctx = ctx;
  int rc = guard(ctx, [&] {
    CK(cudaSetDevice(ctx->device));
    load_residual_model(m, path, base);
    return VG_OK;
  });
  if (rc) {
    if (m->arena) cudaFree(m->arena);
    delete m;
    return rc;
  }
  live_add(m);
  *out = m;
  return VG_OK;
}

namespace {
// One ResidualLM position (step_record_submit, src/acoustic.rs:851-900): with
// fsq_applied, FSQ(BaseLM hidden) (record_fsq :921-944) becomes the LM state,
// else the raw BaseLM hidden does (a text-prefix position); the fusion
// projection of [LM state | current acoustic embedding] (record_fusion
// :946-966) is the input of the ResidualLM layers (record_residual_lm
// :968-1035). The inputs are copied in place first: the BaseLM hidden into
// res_base (FSQ positions) or straight into the LM state, the embedding (or
// zeros) after it. With the step kernel the whole position is one launch (FSQ
// and fusion are its first phases); otherwise standalone kernels run them.
void residual_enqueue(vg_stream *s, const float *base, const float *embed, bool fsq, cudaMemcpyKind kind) {
  vg_model *m = s->m;
  const uint32_t H = m->cfg.embedding_length, LAT = m->acoustic.fsq_latent_dim;
  const size_t bytes = (size_t)H * 4;
  CK(cudaMemcpyAsync(fsq ? s->res_base : s->fuse_in, base, bytes, kind, s->st));
  if (embed)
    CK(cudaMemcpyAsync(s->fuse_in + H, embed, bytes, kind, s->st));
  else
    CK(cudaMemsetAsync(s->fuse_in + H, 0, bytes, s->st));  // zero_embed
  if (s->use_step) {
    launch_residual_step(s, fsq);
    return;
  }
  if (fsq) {
    CK(run_matvec(s->fsq_in_p, s->st, false));
    fsq_quantize_kernel<<<(LAT + 255) / 256, 256, 0, s->st>>>(s->fsq_lat, LAT, m->acoustic.fsq_scale);
    CK(cudaGetLastError());
    CK(run_matvec(s->fsq_out_p, s->st, false));
    CK(cudaMemcpyAsync(s->fuse_in, s->fsq_res, bytes, cudaMemcpyDeviceToDevice, s->st));
  }
  CK(run_matvec(s->fuse_p, s->st, false));
  CK(cudaMemcpyAsync(s->hid_a, s->fused, bytes, cudaMemcpyDeviceToDevice, s->st));
  launch_step(s, false, false);
}
}  // namespace

int vg_residual_step(vg_stream *s, const float *dev_base_hidden, const float *dev_embed, int fsq_applied) {
  if (!live(s)) return VG_ESTATE;
  if (!dev_base_hidden) return VG_EINVAL;
  if (!s->m->residual) return VG_EINVAL;
  return guard(s->m->ctx, [&] {
    check_step(s);
    CK(cudaSetDevice(s->m->ctx->device));
    residual_enqueue(s, dev_base_hidden, dev_embed, fsq_applied != 0, cudaMemcpyDeviceToDevice);
    return VG_OK;
  });
}

int vg_residual_step_host(vg_stream *s, const float *base_hidden, const float *embed, int fsq_applied) {
  if (!live(s)) return VG_ESTATE;
  if (!base_hidden) return VG_EINVAL;
  if (!s->m->residual) return VG_EINVAL;
  return guard(s->m->ctx, [&] {
    check_step(s);
    CK(cudaSetDevice(s->m->ctx->device));
    residual_enqueue(s, base_hidden, embed, fsq_applied != 0, cudaMemcpyHostToDevice);
    CK(cudaStreamSynchronize(s->st));  // the host buffers may be reused on return
    return VG_OK;
  });
}

int vg_residual_state(const vg_stream *s, int which, const float **dev) {
  if (!live(s)) return VG_ESTATE;
  if (!dev || !s->m->residual) return VG_EINVAL;
  switch (which) {
    case VG_RESIDUAL_FSQ_OUTPUT: *dev = s->fsq_res; return VG_OK;
    case VG_RESIDUAL_FUSED_INPUT: *dev = s->fused; return VG_OK;
    case VG_RESIDUAL_LM_STATE: *dev = s->fuse_in; return VG_OK;
  }
  return VG_EINVAL;
}

int vg_residual_copy_state(vg_stream *s, int which, float *host, size_t n) {
  if (!live(s)) return VG_ESTATE;
  if (!host || !s->m->residual || n > s->m->cfg.embedding_length) return VG_EINVAL;
  const float *dev = nullptr;
  int rc = vg_residual_state(s, which, &dev);
  if (rc) return rc;
  return guard(s->m->ctx, [&] {
    CK(cudaSetDevice(s->m->ctx->device));
    CK(cudaStreamSynchronize(s->st));
    CK(cudaMemcpy(host, dev, n * 4, cudaMemcpyDeviceToHost));
    return VG_OK;
  });
}

int vg_prefill_tokens(vg_stream *s, const uint32_t *tokens, uint32_t n, int want_logits_last) {
  if (!live(s)) return VG_ESTATE;
  if (n == 0) {
    set_err(s->m->ctx, "prefill token list is empty");
    return VG_EINVAL;
  }
  if (!tokens) return VG_EINVAL;
  vg_model *m = s->m;
  bool batched = false;
  int rc = guard(m->ctx, [&] {
    for (uint32_t i = 0; i < n; ++i)
      if (tokens[i] >= m->cfg.vocab_size)
        fail(VG_ERANGE, strf("token id %u is outside vocabulary 0..%u", tokens[i], m->cfg.vocab_size));
    check_step(s);
    if ((uint64_t)s->pos + n > s->max_ctx)
      fail(VG_EFULL, strf("BaseLM KV cache is full at %u tokens; reset or increase --max-context", s->max_ctx));
    if (want_logits_last && m->cfg.vocab_size == 0) fail(VG_EUNSUPPORTED, "this model has no LM head");
    if (n < 2 || !s->use_step) return VG_OK;
    CK(cudaSetDevice(m->ctx->device));
    std::lock_guard<std::mutex> lk(m->batch_mu);
    BatchWork *w = get_batch(m);
    if (!w->why.empty()) return VG_OK;
    // runs of up to 16 consecutive positions, one weight pass each
    for (uint32_t i0 = 0; i0 < n; i0 += kBatchMaxCols) {
      const uint32_t k = std::min<uint32_t>(kBatchMaxCols, n - i0);
      std::vector<BatchCol> cols;
      for (uint32_t j = 0; j < k; ++j) cols.push_back(batch_col(s, j, j + 1 == k ? k : 0u, tokens[i0 + j]));
      batch_launch(*w, cols, {s});
      s->pos += k;
    }
    if (want_logits_last) {
      if (!s->head_planned) {
        if (s->step_head_apart) {
          s->head_plan = s->step_head;
        } else {
          s->head_plan = plan_matvec<Mode::PLAIN, Pro::COPY>(m->out, m->ctx->device, (uint32_t)m->ctx->sms);
          s->head_plan.p.xsrc = s->out_norm;
          s->head_plan.p.out = s->logits;
          s->head_plan.p.alpha = eff_scale(m->cfg.logit_scale);
          s->head_plan.p.ctrl = s->ctrl;
        }
        s->head_planned = true;
      }
      CK(run_matvec(s->head_plan, s->st, false));
    }
    s->logits_valid = want_logits_last != 0;
    batched = true;
    return VG_OK;
  });
  if (rc || batched) return rc;
  // one decode step per token: a stream on the per-kernel program, a model the
  // batched kernel does not take, or a single token
  for (uint32_t i = 0; i < n; ++i) {
    rc = vg_decode_token(s, tokens[i], (i + 1 == n) ? want_logits_last : 0);
    if (rc) return rc;
  }
  return VG_OK;
}

int vg_model_batch_columns(vg_model *m, uint32_t *max_columns) {
  if (!live(m)) return VG_ESTATE;
  if (!max_columns) return VG_EINVAL;
  return guard(m->ctx, [&] {
    CK(cudaSetDevice(m->ctx->device));
    std::lock_guard<std::mutex> lk(m->batch_mu);
    BatchWork *w = get_batch(m);
    *max_columns = w->why.empty() ? kBatchMaxCols : 0u;
    if (!w->why.empty()) set_err(m->ctx, "batched step kernel unavailable: " + w->why);
    return VG_OK;
  });
}

int vg_stream_output(const vg_stream *s, const float **dev) {
  if (!live(s)) return VG_ESTATE;
  if (!dev) return VG_EINVAL;
  *dev = s->out_norm;
  return VG_OK;
}

int vg_stream_logits(const vg_stream *s, const float **dev) {
  if (!live(s)) return VG_ESTATE;
  if (!dev) return VG_EINVAL;
  *dev = s->logits;
  return VG_OK;
}

static int copy_out(vg_stream *s, const float *src, float *host, size_t n, size_t limit) {
  return guard(s->m->ctx, [&] {
    if (n > limit) fail(VG_EINVAL, strf("requested %zu floats, buffer holds %zu", n, limit));
    CK(cudaSetDevice(s->m->ctx->device));
    // output block = out_norm then ctrl: one copy brings back the flag too
    const bool with_flag = src == s->out_norm;
    const size_t bytes = with_flag ? (size_t)((uint8_t *)(s->ctrl + kCtrlWords) - (uint8_t *)s->out_norm) : n * 4;
    CK(cudaMemcpyAsync(s->pin_out, src, bytes, cudaMemcpyDeviceToHost, s->st));
    CK(cudaEventRecord(s->ev_done, s->st));
    int rc = host_wait(s->ev_done, 30ull * 1000000000ull);
    if (rc) fail(rc, "output copy did not finish within the timeout");
    if (with_flag) {
      uint32_t flag;
      std::memcpy(&flag, s->pin_out + ((uint8_t *)(s->ctrl + kCtrlErr) - (uint8_t *)s->out_norm), 4);
      if (flag) {
        CK(cudaMemset(s->ctrl + kCtrlErr, 0, 4));
        fail(VG_EDEVICE, strf("a kernel raised device error flag 0x%x", flag));
      }
    }
    std::memcpy(host, s->pin_out, n * 4);
    return VG_OK;
  });
}

int vg_copy_output(vg_stream *s, float *host, size_t n) {
  if (!live(s)) return VG_ESTATE;
  if (!host && n) return VG_EINVAL;
  return copy_out(s, s->out_norm, host, n, s->m->cfg.embedding_length);
}

int vg_copy_outputs(vg_stream *const *streams, int n, float *host, size_t n_each) {
  if (!streams || n <= 0 || (!host && n_each)) return VG_EINVAL;
  for (int i = 0; i < n; ++i)
    if (!live(streams[i])) return VG_ESTATE;
  vg_ctx *ctx = streams[0]->m->ctx;
  return guard(ctx, [&] {
    for (int i = 0; i < n; ++i)
      if (n_each > streams[i]->m->cfg.embedding_length)
        fail(VG_EINVAL, strf("stream %d: requested %zu floats, its output holds %u", i, n_each,
                             streams[i]->m->cfg.embedding_length));
    // every copy is enqueued before the first wait, so the n round trips overlap
    for (int i = 0; i < n; ++i) {
      vg_stream *s = streams[i];
      CK(cudaSetDevice(s->m->ctx->device));
      const size_t bytes = (size_t)((uint8_t *)(s->ctrl + kCtrlWords) - (uint8_t *)s->out_norm);
      CK(cudaMemcpyAsync(s->pin_out, s->out_norm, bytes, cudaMemcpyDeviceToHost, s->st));
      CK(cudaEventRecord(s->ev_done, s->st));
    }
    for (int i = 0; i < n; ++i) {
      const int rc = host_wait(streams[i]->ev_done, 30ull * 1000000000ull);
      if (rc) fail(rc, strf("stream %d: output copy did not finish within the timeout", i));
    }
    int first_bad = -1;
    uint32_t bad_flag = 0;
    for (int i = 0; i < n; ++i) {
      vg_stream *s = streams[i];
      uint32_t flag;
      std::memcpy(&flag, s->pin_out + ((uint8_t *)(s->ctrl + kCtrlErr) - (uint8_t *)s->out_norm), 4);
      if (flag) {
        CK(cudaSetDevice(s->m->ctx->device));
        CK(cudaMemset(s->ctrl + kCtrlErr, 0, 4));
        if (first_bad < 0) {
          first_bad = i;
          bad_flag = flag;
        }
      }
      std::memcpy(host + (size_t)i * n_each, s->pin_out, n_each * 4);
    }
    if (first_bad >= 0)
      fail(VG_EDEVICE, strf("stream %d: a kernel raised device error flag 0x%x", first_bad, bad_flag));
    return VG_OK;
  });
}

int vg_copy_logits(vg_stream *s, float *host, size_t n) {
  if (!live(s)) return VG_ESTATE;
  if (!host && n) return VG_EINVAL;
  return copy_out(s, s->logits, host, n, s->m->cfg.vocab_size);
}

int vg_stream_sync(vg_stream *s, uint64_t timeout_ns) {
  if (!live(s)) return VG_ESTATE;
  return guard(s->m->ctx, [&] {
    CK(cudaSetDevice(s->m->ctx->device));
    return sync_stream(s, timeout_ns, true);
  });
}

int vg_step_result_get(vg_stream *s, uint32_t top_k, vg_step_result *res, vg_top_logit *top) {
  if (!live(s)) return VG_ESTATE;
  if (!res || (top_k && !top)) return VG_EINVAL;
  const uint32_t H = s->m->cfg.embedding_length, V = s->m->cfg.vocab_size;
  std::vector<float> h(H);
  int rc = vg_copy_output(s, h.data(), H);
  if (rc) return rc;
  double sum = 0, sq = 0;
  for (float x : h) {
    sum += (double)x;
    sq += (double)x * (double)x;
  }
  res->position = s->pos ? s->pos - 1 : 0;
  res->final_hidden_checksum = sum;
  res->final_hidden_l2 = std::sqrt(sq);
  res->n_top = 0;
  if (top_k) {
    if (!s->logits_valid) {
      set_err(s->m->ctx, "the last step did not compute logits");
      return VG_ESTATE;
    }
    std::vector<float> lg(V);
    rc = vg_copy_logits(s, lg.data(), V);
    if (rc) return rc;
    rc = vg_top_k_logits(lg.data(), V, top_k, top, &res->n_top);
    if (rc) return rc;
  }
  return VG_OK;
}

int vg_benchmark(vg_stream *s, uint32_t token, uint32_t warmup, uint32_t iterations, int want_logits,
                 vg_benchmark_result *res) {
  if (!live(s)) return VG_ESTATE;
  if (!res) return VG_EINVAL;
  return guard(s->m->ctx, [&] {
    if (iterations == 0) fail(VG_EINVAL, "benchmark iterations must be > 0");
    const uint64_t needed = (uint64_t)warmup + iterations;
    if (needed > s->max_ctx)
      fail(VG_EFULL, strf("benchmark needs %llu context positions but --max-context is %u",
                          (unsigned long long)needed, s->max_ctx));
    int rc = vg_stream_reset(s);
    if (rc) return rc;
    for (uint32_t i = 0; i < warmup; ++i)
      if ((rc = vg_decode_token(s, token, want_logits))) return rc;
    std::vector<cudaEvent_t> ev(iterations + 1);
    for (auto &e : ev) CK(cudaEventCreate(&e));
    CK(cudaEventRecord(ev[0], s->st));
    for (uint32_t i = 0; i < iterations; ++i) {
      if ((rc = vg_decode_token(s, token, want_logits))) break;
      CK(cudaEventRecord(ev[i + 1], s->st));
    }
    if (!rc) rc = sync_stream(s, 120ull * 1000000000ull, true);
    double sum = 0, mn = 1e30, mx = 0;
    if (!rc)
      for (uint32_t i = 0; i < iterations; ++i) {
        float ms = 0;
        CK(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
        sum += ms;
        mn = std::min<double>(mn, ms);
        mx = std::max<double>(mx, ms);
      }
    for (auto &e : ev) cudaEventDestroy(e);
    if (rc) return rc;
    res->iterations = iterations;
    res->token_id = token;
    res->mean_ms = sum / iterations;
    res->min_ms = mn;
    res->max_ms = mx;
    res->tokens_per_second = 1000.0 / res->mean_ms;
    return VG_OK;
  });
}

int vg_stream_profile_step(vg_stream *s, uint32_t token, int want_logits, vg_kernel_time *out, uint32_t capacity,
                           uint32_t *n_out) {
  if (!live(s)) return VG_ESTATE;
  if (!n_out || (!out && capacity)) return VG_EINVAL;
  return guard(s->m->ctx, [&] {
    if (token >= s->m->cfg.vocab_size)
      fail(VG_ERANGE, strf("token id %u is outside vocabulary 0..%u", token, s->m->cfg.vocab_size));
    check_step(s);
    CK(cudaSetDevice(s->m->ctx->device));
    std::vector<Launch> prog;
    build_program(s, true, want_logits != 0, prog);
    uint8_t *slot = staging_slot(s);
    std::memcpy(slot, &token, 4);
    CK(cudaMemcpyAsync(s->ctrl + kCtrlToken, slot, 4, cudaMemcpyHostToDevice, s->st));
    CK(cudaEventRecord(staging_event(s), s->st));
    std::vector<cudaEvent_t> ev(prog.size() + 1);
    for (auto &e : ev) CK(cudaEventCreate(&e));
    cudaError_t err = cudaEventRecord(ev[0], s->st);
    for (size_t i = 0; i < prog.size() && err == cudaSuccess; ++i) {
      err = prog[i].fn(s->st, false);
      if (err == cudaSuccess) err = cudaEventRecord(ev[i + 1], s->st);
    }
    const uint32_t pos = s->pos;
    s->pos += 1;
    s->logits_valid = want_logits != 0;
    int rc = err == cudaSuccess ? sync_stream(s, 60ull * 1000000000ull, true) : VG_ECUDA;
    uint32_t n = 0;
    if (rc == VG_OK) {
      for (size_t i = 0; i < prog.size() && n < capacity; ++i, ++n) {
        float ms = 0;
        CK(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
        vg_kernel_time &k = out[n];
        std::memset(&k, 0, sizeof k);
        snprintf(k.name, sizeof k.name, "%s", prog[i].name);
        k.layer = prog[i].layer;
        k.ms = ms;
        k.bytes = prog[i].per_position ? prog[i].bytes * (uint64_t)(pos + 1) : prog[i].bytes;
      }
    }
    for (auto &e : ev) cudaEventDestroy(e);
    if (err != cudaSuccess) fail(VG_ECUDA, strf("kernel launch failed: %s", cudaGetErrorString(err)));
    *n_out = n;
    return rc;
  });
}

int vg_decode_batch(vg_stream *const *streams, int n, const uint32_t *tokens) {
  if (!streams || !tokens || n <= 0 || n > 16) return VG_EINVAL;
  for (int i = 0; i < n; ++i)
    if (!live(streams[i])) return VG_ESTATE;
  vg_model *m = streams[0]->m;
  return guard(m->ctx, [&] {
    // all streams are checked before any is advanced, so a failure leaves every position unchanged
    std::set<const vg_stream *> seen;
    for (int i = 0; i < n; ++i) {
      vg_stream *s = streams[i];
      if (s->m != m) fail(VG_EINVAL, "vg_decode_batch: streams of different models");
      if (!seen.insert(s).second) fail(VG_EINVAL, "vg_decode_batch: a stream appears twice");
      if (tokens[i] >= m->cfg.vocab_size)
        fail(VG_ERANGE, strf("token id %u is outside vocabulary 0..%u", tokens[i], m->cfg.vocab_size));
      check_step(s);
    }
    CK(cudaSetDevice(m->ctx->device));
    bool all_step = n >= 2;
    for (int i = 0; i < n; ++i) all_step = all_step && streams[i]->use_step;
    if (all_step) {
      // one launch of the batched kernel: one weight pass for every stream
      std::lock_guard<std::mutex> lk(m->batch_mu);
      BatchWork *w = get_batch(m);
      if (w->why.empty()) {
        std::vector<BatchCol> cols;
        std::vector<vg_stream *> ss;
        for (int i = 0; i < n; ++i) {
          cols.push_back(batch_col(streams[i], 0u, 1u, tokens[i]));
          ss.push_back(streams[i]);
        }
        batch_launch(*w, cols, ss);
        for (vg_stream *s : ss) {
          s->pos += 1;
          s->logits_valid = false;
        }
        return VG_OK;
      }
    }
    // one step per stream, each on its own CUDA stream (the weights are read once per stream)
    for (int i = 0; i < n; ++i) {
      vg_stream *s = streams[i];
      uint8_t *slot = staging_slot(s);
      std::memcpy(slot, &tokens[i], 4);
      CK(cudaMemcpyAsync(s->ctrl + kCtrlToken, slot, 4, cudaMemcpyHostToDevice, s->st));
      CK(cudaEventRecord(staging_event(s), s->st));
      launch_step(s, true, false);
    }
    return VG_OK;
  });
}

// ---- kernel-level entry points --------------------------------------------
static std::mutex g_kctrl_mu;
static std::map<int, uint32_t *> g_kctrl;  // per-device control words for kernel-level calls

static uint32_t *kernel_ctrl() {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> l(g_kctrl_mu);
  uint32_t *&p = g_kctrl[dev];
  if (!p) {
    CK(cudaMalloc(&p, kCtrlWords * 4));
    CK(cudaMemset(p, 0, kCtrlWords * 4));
  }
  return p;
}

// Scratch of vg_k_attention_noalloc: merge tickets, then per-cluster partials.
// A file-scope device array, zero when the module loads; its address is looked
// up once per device and cached.
constexpr uint32_t kNoAllocScratchBytes = VG_K_ATTENTION_NOALLOC_TICKET_BYTES + VG_K_ATTENTION_NOALLOC_PARTIAL_BYTES;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

static uint8_t *noalloc_scratch(int dev) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static uint8_t *addr[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) fail(VG_EDEVICE, strf("device %d out of range", dev));
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void *a = nullptr;
    CK(cudaGetSymbolAddress(&a, g_noalloc_scratch));
    addr[dev] = (uint8_t *)a;
  }
  return addr[dev];
}

static int kguard(const std::function<void()> &f) {
  try {
    f();
    return VG_OK;
  } catch (const Error &e) {
    return e.code;
  }
}

int vg_k_packed_bytes(int dtype, uint32_t rows, uint32_t cols, uint64_t *bytes) {
  if (!bytes || rows == 0 || cols == 0) return VG_EINVAL;
  if (dtype == VG_FORMAT_Q8_0 && cols % 32 == 0) *bytes = packed_bytes(GGML_Q8_0, rows, cols);
  else if (dtype == VG_FORMAT_F16 && cols % 8 == 0) *bytes = packed_bytes(GGML_F16, rows, cols);
  else return VG_EUNSUPPORTED;
  return VG_OK;
}

int vg_k_repack(int dtype, const void *gguf_bytes, uint32_t rows, uint32_t cols, void *packed, void *cuda_stream) {
  uint64_t b;
  int rc = vg_k_packed_bytes(dtype, rows, cols, &b);
  if (rc) return rc;
  if (!gguf_bytes || !packed) return VG_EINVAL;
  return kguard([&] {
    cudaStream_t st = (cudaStream_t)cuda_stream;
    CK(cudaMemsetAsync(packed, 0, b, st));
    const TileGeom g{rows, cols, dtype == VG_FORMAT_Q8_0 ? 1u : 0u};
    repack_kernel<<<std::min<uint32_t>(rows, 65535u), 256, 0, st>>>((const uint8_t *)gguf_bytes, rows, g,
                                                                     (uint8_t *)packed, kPermIdentity, 0, 0);
    CK(cudaGetLastError());
  });
}

int vg_k_matvec(int dtype, const void *packed, uint32_t rows, uint32_t cols, const float *x, float *y, float alpha,
                void *cuda_stream) {
  uint64_t b;
  int rc = vg_k_packed_bytes(dtype, rows, cols, &b);
  if (rc) return rc;
  if (!packed || !x || !y) return VG_EINVAL;
  return kguard([&] {
    int dev = 0, sms = 0;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    DevMat m = make_mat(rows, cols, dtype == VG_FORMAT_Q8_0 ? GGML_Q8_0 : GGML_F16);
    m.w = (uint8_t *)packed;
    MvPlan pl = plan_matvec<Mode::PLAIN, Pro::COPY>(m, dev, (uint32_t)sms);
    pl.p.xsrc = x;
    pl.p.out = y;
    pl.p.alpha = alpha;
    pl.p.ctrl = kernel_ctrl();
    CK(run_matvec(pl, (cudaStream_t)cuda_stream, false));
  });
}

int vg_k_embedding(int dtype, const void *packed, uint32_t rows, uint32_t cols, uint32_t row, float alpha,
                   float *out, void *cuda_stream) {
  uint64_t b;
  int rc = vg_k_packed_bytes(dtype, rows, cols, &b);
  if (rc) return rc;
  if (!packed || !out) return VG_EINVAL;
  if (row >= rows) return VG_ERANGE;
  return kguard([&] {
    const TileGeom g{rows, cols, dtype == VG_FORMAT_Q8_0 ? 1u : 0u};
    embedding_kernel<<<(cols + 255) / 256, 256, 0, (cudaStream_t)cuda_stream>>>(
        (const uint8_t *)packed, g, nullptr, row, alpha, out, kernel_ctrl() + kCtrlErr);
    CK(cudaGetLastError());
  });
}

int vg_k_residual_rmsnorm(float *hidden, const float *branch, const float *w, uint32_t n, float eps, float scale,
                          float *y, void *cuda_stream) {
  if (!hidden || !w || !y || n == 0) return VG_EINVAL;
  return kguard([&] {
    residual_rmsnorm_kernel<<<1, std::min<uint32_t>(1024u, round_up(n, 32)), 0, (cudaStream_t)cuda_stream>>>(
        hidden, branch, w, n, eps, scale, y, nullptr, 0);
    CK(cudaGetLastError());
  });
}

int vg_k_attention(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, uint32_t heads,
                   uint32_t kv_heads, uint32_t head_dim, uint32_t ctx, uint32_t position, float *out,
                   void *cuda_stream) {
  if (!q || !k_cache || !v_cache || !out || !heads || !kv_heads || heads % kv_heads || position >= ctx)
    return VG_EINVAL;
  if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256) return VG_EUNSUPPORTED;
  return kguard([&] {
    cudaStream_t st = (cudaStream_t)cuda_stream;
    int dev = 0;
    CK(cudaGetDevice(&dev));
    const uint32_t G = heads / kv_heads;
    AttnParams ap{};
    plan_attention(ctx, ap.nsplit, ap.chunk_cap);
    const size_t part_bytes = (size_t)kv_heads * (ap.nsplit / kAttnCluster) * G * (head_dim + 2) * 4;
    void *scratch = nullptr;
    CK(cudaMallocAsync(&scratch, round_up_sz(part_bytes, 256) + (size_t)kv_heads * G * 4, st));
    uint32_t *tickets = (uint32_t *)((uint8_t *)scratch + round_up_sz(part_bytes, 256));
    CK(cudaMemsetAsync(tickets, 0, (size_t)kv_heads * G * 4, st));
    ap.q = q;
    ap.kc = (const __half *)k_cache;
    ap.vc = (const __half *)v_cache;
    ap.out = out;
    ap.part = (float *)scratch;
    ap.tickets = tickets;
    ap.heads = heads;
    ap.kv_heads = kv_heads;
    ap.ctx = ctx;
    ap.scale = 1.0f / sqrtf((float)head_dim);
    ap.fixed_pos = position;
    ap.ctrl = nullptr;
    const AttnFn fn = pick_attention(head_dim);
    const uint32_t smem = attention_smem_bytes(G, head_dim, ap.chunk_cap);
    ensure_smem((const void *)fn, dev, smem);
    cudaError_t e = launch_ex(fn, dim3(ap.nsplit, kv_heads), dim3(kAttnThreads), smem, st, false, kAttnCluster, ap);
    cudaError_t e2 = cudaFreeAsync(scratch, st);
    CK(e);
    CK(e2);
  });
}

int vg_k_attention_noalloc(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, uint32_t heads,
                           uint32_t kv_heads, uint32_t head_dim, uint32_t ctx, uint32_t position, float *out,
                           void *cuda_stream) {
  if (!q || !k_cache || !v_cache || !out || !heads || !kv_heads || heads % kv_heads || position >= ctx)
    return VG_EINVAL;
  if (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256) return VG_EUNSUPPORTED;
  const uint32_t G = heads / kv_heads;
  AttnParams ap{};
  plan_attention(ctx, ap.nsplit, ap.chunk_cap);
  const uint64_t part_bytes = (uint64_t)kv_heads * (ap.nsplit / kAttnCluster) * G * (head_dim + 2) * 4;
  if (part_bytes > VG_K_ATTENTION_NOALLOC_PARTIAL_BYTES || (uint64_t)heads * 4 > VG_K_ATTENTION_NOALLOC_TICKET_BYTES)
    return VG_ERANGE;
  return kguard([&] {
    cudaStream_t st = (cudaStream_t)cuda_stream;
    int dev = 0;
    CK(cudaGetDevice(&dev));
    uint8_t *scratch = noalloc_scratch(dev);
    uint32_t *tickets = (uint32_t *)scratch;
    CK(cudaMemsetAsync(tickets, 0, (size_t)heads * 4, st));
    ap.q = q;
    ap.kc = (const __half *)k_cache;
    ap.vc = (const __half *)v_cache;
    ap.out = out;
    ap.part = (float *)(scratch + VG_K_ATTENTION_NOALLOC_TICKET_BYTES);
    ap.tickets = tickets;
    ap.heads = heads;
    ap.kv_heads = kv_heads;
    ap.ctx = ctx;
    ap.scale = 1.0f / sqrtf((float)head_dim);
    ap.fixed_pos = position;
    ap.ctrl = nullptr;
    const AttnFn fn = pick_attention(head_dim);
    const uint32_t smem = attention_smem_bytes(G, head_dim, ap.chunk_cap);
    ensure_smem((const void *)fn, dev, smem);
    CK(launch_ex(fn, dim3(ap.nsplit, kv_heads), dim3(kAttnThreads), smem, st, false, kAttnCluster, ap));
  });
}

}  // extern "C"
