// gsvdec_api.cu -- the C ABI (include/gsvdec.h): weight loading and packing
// (Decoder::load), the per-call layer schedule (Decoder::forward) and the
// workspace.  Host code only; kernels live in tapconv_*.cu / misc_kernels.cu.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <algorithm>
#include <array>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <atomic>
#include <vector>

#include "../../include/gsvdec.h"
#include "gsv_kernels.h"
#include "gsv_pdl.cuh"
#include "safetensors.h"

namespace gsv {
namespace {

thread_local std::string g_last_error;

int set_err(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define CUDA_TRY(expr)                                                                 \
  do {                                                                                 \
    cudaError_t e_ = (expr);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return set_err(e_ == cudaErrorMemoryAllocation ? GSV_E_OOM : GSV_E_CUDA,         \
                     "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                     __LINE__);                                                        \
  } while (0)

#define GSV_TRY(expr)          \
  do {                         \
    int rc_ = (expr);          \
    if (rc_ != GSV_OK) return rc_; \
  } while (0)

// Allocation-failure hook (gsvdec_set_alloc_fail_after): while the budget is
// >= 0, each device allocation of the library consumes one unit and fails
// with cudaErrorMemoryAllocation (reported as GSV_E_OOM) once none is left.
// -1 (the default) injects nothing.
std::atomic<int> g_alloc_budget{-1};

cudaError_t dev_malloc_raw(void** p, size_t bytes) {
  *p = nullptr;
  int b = g_alloc_budget.load();
  while (b >= 0) {
    if (b == 0) return cudaErrorMemoryAllocation;
    if (g_alloc_budget.compare_exchange_weak(b, b - 1)) break;
  }
  const cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();  // not sticky: keep it out of later launch checks
    *p = nullptr;
  }
  return e;
}

template <typename T>
cudaError_t dev_malloc(T** p, size_t bytes) {
  void* v = nullptr;
  const cudaError_t e = dev_malloc_raw(&v, bytes);
  *p = static_cast<T*>(v);
  return e;
}

// ---------------------------------------------------------------------------
// Host-side model, following Decoder::load (src/models/sovits_decoder.rs:231-293).

struct HostConv {
  std::string name;      // dec.* prefix of the layer
  std::vector<float> w;  // folded weight, the tensor's own layout [d0, d1, K]
  std::vector<float> b;  // bias or empty
  int d0 = 0, d1 = 0, K = 0;
  int pad = 0, dil = 1, stride = 1;
  // Where w comes from: the plain weight, or (src_g set) the weight-norm pair
  // v = src_w, g = src_g.  Validated at load; converted and folded by
  // materialize(), in parallel over all convs.
  const gsvdec_tensor* src_w = nullptr;
  const gsvdec_tensor* src_g = nullptr;
};

struct HostModel {
  HostConv pre, post, cond;
  bool has_cond = false;
  std::vector<HostConv> ups;  // weight [Cin, Cout, K]
  struct RB {
    std::vector<HostConv> c1, c2;
  };
  std::vector<RB> rbs;
};

float half_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }
float bf16_to_float(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

struct TensorMap {
  std::map<std::string, const gsvdec_tensor*> m;
  const gsvdec_tensor* get(const std::string& k) const {
    auto it = m.find(k);
    return it == m.end() ? nullptr : it->second;
  }
};

int64_t numel(const gsvdec_tensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}

int check_data(const gsvdec_tensor* t) {
  if (!t->data && numel(t)) return set_err(GSV_E_INVALID_ARG, "tensor %s has no data", t->name);
  if (t->dtype != GSV_DTYPE_F32 && t->dtype != GSV_DTYPE_F16 && t->dtype != GSV_DTYPE_BF16)
    return set_err(GSV_E_DTYPE, "tensor %s: unsupported dtype %d", t->name, t->dtype);
  return GSV_OK;
}

// Converts a checked tensor to fp32 (cannot fail: check_data ran first).
void convert_f32(const gsvdec_tensor* t, float* out) {
  const int64_t n = numel(t);
  switch (t->dtype) {
    case GSV_DTYPE_F32:
      memcpy(out, t->data, sizeof(float) * (size_t)n);
      return;
    case GSV_DTYPE_F16: {
      const uint16_t* p = static_cast<const uint16_t*>(t->data);
      for (int64_t i = 0; i < n; ++i) out[i] = half_to_float(p[i]);
      return;
    }
    default: {
      const uint16_t* p = static_cast<const uint16_t*>(t->data);
      for (int64_t i = 0; i < n; ++i) out[i] = bf16_to_float(p[i]);
      return;
    }
  }
}

int to_f32(const gsvdec_tensor* t, std::vector<float>& out) {
  GSV_TRY(check_data(t));
  out.resize((size_t)numel(t));
  convert_f32(t, out.data());
  return GSV_OK;
}

// Runs f(0) .. f(n - 1) on up to hardware_concurrency host threads (the
// calling thread included).  f must not fail or touch the thread-local error.
template <typename F>
void parallel_for(size_t n, F&& f) {
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const size_t nt = std::min<size_t>(std::min<size_t>(hw, 32), n);
  if (nt <= 1) {
    for (size_t i = 0; i < n; ++i) f(i);
    return;
  }
  std::atomic<size_t> next{0};
  auto work = [&] {
    for (size_t i; (i = next.fetch_add(1, std::memory_order_relaxed)) < n;) f(i);
  };
  std::vector<std::thread> pool;
  pool.reserve(nt - 1);
  for (size_t t = 1; t < nt; ++t) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
}

// Plain conv: "<pfx>.weight" [O, I, K], optional "<pfx>.bias"; pad (K-1)/2
// (src/models/sovits_decoder.rs:295-321, 356-383).
int load_plain(const TensorMap& tm, const std::string& pfx, HostConv& c) {
  c.name = pfx;
  const gsvdec_tensor* w = tm.get(pfx + ".weight");
  if (!w) return set_err(GSV_E_MISSING_KEY, "Key '%s.weight' not found in state dict", pfx.c_str());
  if (w->ndim != 3) return set_err(GSV_E_SHAPE, "%s.weight must be 3-d", pfx.c_str());
  GSV_TRY(check_data(w));
  c.src_w = w;
  c.src_g = nullptr;
  c.d0 = (int)w->shape[0];
  c.d1 = (int)w->shape[1];
  c.K = (int)w->shape[2];
  if (const gsvdec_tensor* b = tm.get(pfx + ".bias")) {
    if (numel(b) != c.d0) return set_err(GSV_E_SHAPE, "%s.bias must have %d values", pfx.c_str(), c.d0);
    GSV_TRY(to_f32(b, c.b));
  }
  c.pad = (c.K - 1) / 2;
  return GSV_OK;
}

// Weight-norm conv: w = g * v / ||v||, norm over dims (1, 2) of each dim-0
// slice, folded once at load (src/utils/weights.rs:589-614).
int load_wn(const TensorMap& tm, const std::string& pfx, HostConv& c) {
  c.name = pfx;
  const gsvdec_tensor* v = tm.get(pfx + ".weight_v");
  const gsvdec_tensor* g = tm.get(pfx + ".weight_g");
  if (!v) return set_err(GSV_E_MISSING_KEY, "Key '%s.weight_v' not found in state dict", pfx.c_str());
  if (!g) return set_err(GSV_E_MISSING_KEY, "Key '%s.weight_g' not found in state dict", pfx.c_str());
  if (v->ndim != 3) return set_err(GSV_E_SHAPE, "%s.weight_v must be 3-d", pfx.c_str());
  c.d0 = (int)v->shape[0];
  c.d1 = (int)v->shape[1];
  c.K = (int)v->shape[2];
  if (numel(g) != c.d0)
    return set_err(GSV_E_SHAPE, "%s.weight_g must hold %d values (one per dim-0 slice)", pfx.c_str(), c.d0);
  GSV_TRY(check_data(v));
  GSV_TRY(check_data(g));
  c.src_w = v;
  c.src_g = g;
  if (const gsvdec_tensor* b = tm.get(pfx + ".bias")) GSV_TRY(to_f32(b, c.b));
  c.pad = (c.K - 1) / 2;
  return GSV_OK;
}

// The fp32 weight of a loaded conv: the plain weight converted, or the
// weight-norm fold w = g * v / ||v||, the norm over dims (1, 2) of each dim-0
// slice accumulated in double (src/utils/weights.rs:589-614).
void materialize(HostConv& c) {
  if (!c.src_w) return;
  c.w.resize((size_t)numel(c.src_w));
  convert_f32(c.src_w, c.w.data());
  if (c.src_g) {
    std::vector<float> gg((size_t)numel(c.src_g));
    convert_f32(c.src_g, gg.data());
    const size_t per = (size_t)c.d1 * c.K;
    for (int o = 0; o < c.d0; ++o) {
      float* row = c.w.data() + (size_t)o * per;
      double ss = 0.0;
      for (size_t j = 0; j < per; ++j) ss += (double)row[j] * row[j];
      const float norm = (float)std::sqrt(ss);
      for (size_t j = 0; j < per; ++j) row[j] = (row[j] / norm) * gg[o];
    }
  }
  c.src_w = c.src_g = nullptr;
}

void materialize_all(const std::vector<HostConv*>& cs) {
  parallel_for(cs.size(), [&](size_t i) { materialize(*cs[i]); });
}

int load_model(const gsvdec_tensor* ts, int n, HostModel& m) {
  TensorMap tm;
  for (int i = 0; i < n; ++i) {
    if (!ts[i].name) return set_err(GSV_E_INVALID_ARG, "tensor %d has no name", i);
    if (ts[i].ndim < 1 || ts[i].ndim > 4)
      return set_err(GSV_E_SHAPE, "tensor %s: ndim %d out of range", ts[i].name, ts[i].ndim);
    tm.m[ts[i].name] = &ts[i];
  }
  GSV_TRY(load_plain(tm, "dec.conv_pre", m.pre));
  GSV_TRY(load_plain(tm, "dec.conv_post", m.post));
  if (tm.get("dec.cond.weight")) {
    GSV_TRY(load_plain(tm, "dec.cond", m.cond));
    m.has_cond = true;
    if (m.cond.K != 1) return set_err(GSV_E_SHAPE, "dec.cond.weight must have kernel size 1");
    if (m.cond.d0 != m.pre.d0)
      return set_err(GSV_E_SHAPE, "dec.cond output width %d != conv_pre width %d", m.cond.d0, m.pre.d0);
  }
  // Strides are training config: [10, 8, 2, 2, 2], fallback 2 (:252-270).
  static const int kRates[5] = {10, 8, 2, 2, 2};
  int C = m.pre.d0;
  for (int i = 0; i < 10; ++i) {
    const std::string pfx = "dec.ups." + std::to_string(i);
    if (!tm.get(pfx + ".weight_v")) continue;
    HostConv u;
    GSV_TRY(load_wn(tm, pfx, u));
    const int idx = (int)m.ups.size();
    u.stride = idx < 5 ? kRates[idx] : 2;
    if (u.K < u.stride) return set_err(GSV_E_SHAPE, "%s: kernel %d shorter than stride %d", pfx.c_str(), u.K, u.stride);
    u.pad = (u.K - u.stride) / 2;  // (:564)
    if (u.d0 != C) return set_err(GSV_E_SHAPE, "%s: input width %d != %d", pfx.c_str(), u.d0, C);
    C = u.d1;
    m.ups.push_back(std::move(u));
  }
  // ResBlock1: k = [3,7,11][rb % 3], convs1 dilation [1,3,5][i] (pad d(k-1)/2),
  // convs2 dilation 1 (pad (k-1)/2) (src/models/sovits_decoder.rs:146-194).
  static const int kKs[3] = {3, 7, 11}, kDil[3] = {1, 3, 5};
  for (int r = 0; r < 15; ++r) {
    const std::string pfx = "dec.resblocks." + std::to_string(r);
    if (!tm.get(pfx + ".convs1.0.weight_v")) continue;
    HostModel::RB rb;
    for (int s = 0; s < 2; ++s) {
      for (int j = 0; j < 3; ++j) {
        const std::string cp = pfx + ".convs" + std::to_string(s + 1) + "." + std::to_string(j);
        if (!tm.get(cp + ".weight_v")) continue;
        HostConv c;
        GSV_TRY(load_wn(tm, cp, c));
        const int k = kKs[r % 3];
        if (c.K != k)
          return set_err(GSV_E_SHAPE, "%s: kernel %d disagrees with [3,7,11][rb %% 3] = %d", cp.c_str(), c.K, k);
        if (c.d0 != c.d1) return set_err(GSV_E_SHAPE, "%s: resblock conv must be square", cp.c_str());
        if (s == 0) { c.dil = kDil[j]; c.pad = kDil[j] * (k - 1) / 2; }
        else { c.dil = 1; c.pad = (k - 1) / 2; }
        (s == 0 ? rb.c1 : rb.c2).push_back(std::move(c));
      }
    }
    if (rb.c1.size() != rb.c2.size() || rb.c1.empty())
      return set_err(GSV_E_SHAPE, "%s: convs1 / convs2 counts differ", pfx.c_str());
    m.rbs.push_back(std::move(rb));
  }
  // Resblock widths must match their stage.
  C = m.pre.d0;
  for (size_t i = 0; i < m.ups.size(); ++i) {
    C = m.ups[i].d1;
    for (size_t r = 3 * i; r < std::min(3 * i + 3, m.rbs.size()); ++r)
      if (m.rbs[r].c1[0].d0 != C)
        return set_err(GSV_E_SHAPE, "dec.resblocks.%zu width %d != stage width %d", r, m.rbs[r].c1[0].d0, C);
  }
  if (m.post.d1 != C) return set_err(GSV_E_SHAPE, "dec.conv_post input width %d != %d", m.post.d1, C);
  if (m.post.d0 != 1) return set_err(GSV_E_SHAPE, "dec.conv_post must have one output channel");
  return GSV_OK;
}

// ---------------------------------------------------------------------------
// Host-side flow, following ResidualCouplingBlock::load
// (src/models/sovits_flow.rs:346-368): coupling layers at indices 0..7 that
// carry "<i>.pre.weight"; per layer pre/post (weight-norm pair if present,
// else the plain weight: :225-279), and a WN (:19-109) of in_layers (k, pad
// (k-1)/2, dilation 1), res_skip_layers and an optional cond_layer.

struct HostCoupling {
  HostConv pre, post, cond;
  std::vector<HostConv> in, rs;
  bool has_cond = false;
};

struct HostFlow {
  std::vector<HostCoupling> layers;
};

int load_pre_post(const TensorMap& tm, const std::string& pfx, HostConv& c) {
  if (tm.get(pfx + ".weight_v")) return load_wn(tm, pfx, c);
  return load_plain(tm, pfx, c);
}

int load_flow(const gsvdec_tensor* ts, int n, const std::string& prefix, HostFlow& f) {
  TensorMap tm;
  for (int i = 0; i < n; ++i)
    if (ts[i].name) tm.m[ts[i].name] = &ts[i];
  for (int i = 0; i < 8; ++i) {
    const std::string p = prefix + "." + std::to_string(i);
    if (!tm.get(p + ".pre.weight")) continue;
    HostCoupling c;
    GSV_TRY(load_pre_post(tm, p + ".pre", c.pre));
    GSV_TRY(load_pre_post(tm, p + ".post", c.post));
    for (int j = 0; tm.get(p + ".enc.in_layers." + std::to_string(j) + ".weight_v"); ++j) {
      HostConv a;
      GSV_TRY(load_wn(tm, p + ".enc.in_layers." + std::to_string(j), a));
      c.in.push_back(std::move(a));
    }
    for (size_t j = 0; j < c.in.size(); ++j) {
      HostConv r;
      GSV_TRY(load_wn(tm, p + ".enc.res_skip_layers." + std::to_string(j), r));
      c.rs.push_back(std::move(r));
    }
    if (tm.get(p + ".enc.cond_layer.weight_v")) {
      GSV_TRY(load_wn(tm, p + ".enc.cond_layer", c.cond));
      c.has_cond = true;
    }
    if (c.in.empty()) return set_err(GSV_E_MISSING_KEY, "Key '%s.enc.in_layers.0.weight_v' not found in state dict", p.c_str());
    f.layers.push_back(std::move(c));
  }
  return GSV_OK;
}

// Host-side EncP chains, following EncoderLayer::load and FeedForward::load
// (src/models/sovits_encp.rs:54-96, :348-369): per stack, layers 0, 1, ...
// while "<stack>.ffn_layers.<i>.conv_1.weight" exists, convs with pad (k-1)/2
// (load_conv1d :378-410) and both LayerNorm pairs required.  enc_p.proj is a
// 1x1 conv with pad 0 (:752-771).
struct HostEncpLayer {
  HostConv c1, c2;
  std::vector<float> g1, b1, g2, b2;
};

struct HostEncp {
  std::vector<HostEncpLayer> stacks[3];
  HostConv proj;
  bool has_proj = false;
};

const char* const kEncpStacks[3] = {"enc_p.encoder_ssl", "enc_p.encoder_text", "enc_p.encoder2"};

int load_vec(const TensorMap& tm, const std::string& key, int n, std::vector<float>& v) {
  const gsvdec_tensor* t = tm.get(key);
  if (!t) return set_err(GSV_E_MISSING_KEY, "Key '%s' not found in state dict", key.c_str());
  if (numel(t) != n) return set_err(GSV_E_SHAPE, "%s must have %d values", key.c_str(), n);
  return to_f32(t, v);
}

int load_encp(const gsvdec_tensor* ts, int n, HostEncp& e) {
  TensorMap tm;
  for (int i = 0; i < n; ++i)
    if (ts[i].name) tm.m[ts[i].name] = &ts[i];
  int C = 0;
  for (int s = 0; s < 3; ++s) {
    const std::string p = kEncpStacks[s];
    for (int i = 0; i < 64; ++i) {
      const std::string f = p + ".ffn_layers." + std::to_string(i);
      if (!tm.get(f + ".conv_1.weight")) break;
      HostEncpLayer L;
      GSV_TRY(load_plain(tm, f + ".conv_1", L.c1));
      GSV_TRY(load_plain(tm, f + ".conv_2", L.c2));
      if (L.c2.d0 != L.c1.d1 || L.c2.d1 != L.c1.d0)
        return set_err(GSV_E_SHAPE, "%s: conv_2 [%d,%d] does not invert conv_1 [%d,%d]", f.c_str(), L.c2.d0,
                       L.c2.d1, L.c1.d0, L.c1.d1);
      if (C && L.c1.d1 != C) return set_err(GSV_E_SHAPE, "%s: hidden width %d != %d", f.c_str(), L.c1.d1, C);
      C = L.c1.d1;
      const std::string is = std::to_string(i);
      GSV_TRY(load_vec(tm, p + ".norm_layers_1." + is + ".gamma", C, L.g1));
      GSV_TRY(load_vec(tm, p + ".norm_layers_1." + is + ".beta", C, L.b1));
      GSV_TRY(load_vec(tm, p + ".norm_layers_2." + is + ".gamma", C, L.g2));
      GSV_TRY(load_vec(tm, p + ".norm_layers_2." + is + ".beta", C, L.b2));
      e.stacks[s].push_back(std::move(L));
    }
  }
  if (tm.get("enc_p.proj.weight")) {
    GSV_TRY(load_plain(tm, "enc_p.proj", e.proj));
    if (e.proj.K != 1) return set_err(GSV_E_UNSUPPORTED, "enc_p.proj with kernel %d (1 expected)", e.proj.K);
    if (C && e.proj.d1 != C) return set_err(GSV_E_SHAPE, "enc_p.proj input width %d != %d", e.proj.d1, C);
    if (e.proj.d0 % 2) return set_err(GSV_E_SHAPE, "enc_p.proj has an odd output width %d", e.proj.d0);
    e.proj.pad = 0;
    e.has_proj = true;
  }
  return GSV_OK;
}

// ---------------------------------------------------------------------------
// Packed device form of one conv as a tap GEMM (see gsv_internal.h).

struct GemmConv {
  int Cin = 0, Cout = 0, N = 0, ntaps = 0, off0 = 0, offstep = 1;
  int stride = 1, pad = 0, K = 0;  // ConvT: Q/crop/Lout derive from these
  bool transposed = false;
  bool x3 = false;   // three-piece packing (GSV_MODE_FP32_TC decoder), in the second arena
  size_t w_off = 0;  // byte offset in the weight arena (three-piece: the five small-product blocks)
  size_t w_off2 = 0; // three-piece: the large-product block W0
  size_t b_off = 0;  // float offset in the bias arena
  int Lout(int Lin) const {
    return transposed ? (Lin - 1) * stride + K - 2 * pad : Lin + 2 * pad - (ntaps - 1) * offstep;
  }
  int Q(int Lin) const { return transposed ? (Lout(Lin) + pad - 1) / stride + 1 : Lout(Lin); }
};

// Builds the weight arena.  conv()/convT()/identity() only reserve the bytes
// and record fill jobs; finish() allocates the arena once and runs the jobs in
// parallel.  The HostConv weights a job reads must stay alive (and unmoved)
// until finish(): the loaded model's convs live for the whole create call, and
// temporaries are handed over with conv(HostConv&&).
struct Packer {
  Dt dt;
  bool x3 = false;                      // three-piece bf16 packing (dt BF16)
  size_t size = 0;                      // bytes reserved so far
  std::unique_ptr<uint8_t[]> arena;     // size bytes after finish()
  std::vector<float> biases;

  enum Kind { kConv, kConvT, kIdentity };
  struct Job {
    Kind kind;
    const float* w;  // HostConv layout: conv [N][Cin][K], convT [Cin][Cout][K]
    const int* rows; // conv: packed column n reads weight row rows[n] (NULL: n)
    int Cin, Cout, N, K, stride;
    size_t base;
    size_t base2;    // three-piece: the W0 block
    int j, n0, n1;   // tap j, packed columns [n0, n1)
  };
  std::vector<Job> jobs;
  std::vector<std::pair<size_t, size_t>> gaps;  // alignment padding to zero
  std::vector<std::unique_ptr<std::vector<float>>> owned;
  std::vector<std::unique_ptr<std::vector<int>>> owned_rows;

  size_t esize() const { return dt == Dt::F32 ? 4 : 2; }
  // Packed K entries per input channel: a three-piece conv's first K list
  // is five weight pieces long ([W0 W1 W2 W0 W1] against [X2 X1 X0 X1 X0]);
  // its second (W0 against X0) follows at w_off2.
  int kmul() const { return x3 ? 5 : 1; }
  void reserve_x3_second(GemmConv& g) {
    if (x3) g.w_off2 = reserve((size_t)g.ntaps * g.N * g.Cin * esize());
  }
  size_t reserve(size_t bytes) {
    const size_t r = (size + 1023) / 1024 * 1024;
    if (r > size) gaps.emplace_back(size, r - size);
    size = r + bytes;
    return r;
  }
  // One job per tap and block of about 64k packed elements.
  void add_jobs(Kind kind, const float* w, const GemmConv& g, int Cin, int K, int stride,
                const int* rows = nullptr) {
    const int cols = std::max(1, 65536 / std::max(Cin, 1));
    for (int j = 0; j < g.ntaps; ++j)
      for (int n0 = 0; n0 < g.N; n0 += cols)
        jobs.push_back(Job{kind, w, rows, Cin, g.Cout, g.N, K, stride, g.w_off, g.w_off2, j, n0,
                           std::min(g.N, n0 + cols)});
  }

  GemmConv conv(const HostConv& c) { return conv_from(c, c.w.data()); }
  GemmConv conv(HostConv&& c) {
    owned.push_back(std::make_unique<std::vector<float>>(std::move(c.w)));
    return conv_from(c, owned.back()->data());
  }
  // The conv c with its output rows reordered (packed column n = row rows[n])
  // or truncated to the first d0 rows (d0 below c.d0), reading c's weights in
  // place.
  GemmConv conv_rows(const HostConv& c, std::vector<int> rows, int d0) {
    HostConv view;
    view.d0 = d0; view.d1 = c.d1; view.K = c.K; view.pad = c.pad; view.dil = c.dil;
    if (!c.b.empty())
      for (int n = 0; n < d0; ++n) view.b.push_back(c.b[rows.empty() ? n : rows[n]]);
    const int* map = nullptr;
    if (!rows.empty()) {
      owned_rows.push_back(std::make_unique<std::vector<int>>(std::move(rows)));
      map = owned_rows.back()->data();
    }
    return conv_from(view, c.w.data(), map);
  }
  GemmConv conv_from(const HostConv& c, const float* w, const int* rows = nullptr) {
    GemmConv g;
    g.Cin = c.d1; g.Cout = c.d0; g.N = c.d0; g.ntaps = c.K;
    g.off0 = -c.pad; g.offstep = c.dil; g.pad = c.pad; g.K = c.K; g.x3 = x3;
    g.w_off = reserve((size_t)g.ntaps * g.N * g.Cin * kmul() * esize());
    reserve_x3_second(g);
    add_jobs(kConv, w, g, g.Cin, c.K, 1, rows);
    g.b_off = biases.size();
    for (int n = 0; n < g.Cout; ++n) biases.push_back(c.b.empty() ? 0.0f : c.b[n]);
    return g;
  }
  // Identity [1][C][C]: a ResBlock residual fed through the MMA (bf16 mode).
  size_t identity(int C) {
    GemmConv g;
    g.Cin = C; g.Cout = C; g.N = C; g.ntaps = 1;
    g.w_off = reserve((size_t)C * C * (x3 ? 3 : 1) * esize());
    add_jobs(kIdentity, nullptr, g, C, 1, 1);
    return g.w_off;
  }
  // Polyphase ConvTranspose1d: tap m, column n = phi*Cout + o, channel c holds
  // w[c][o][phi + m*s] (zero past the kernel).
  GemmConv convT(const HostConv& c) {
    GemmConv g;
    g.transposed = true;
    g.Cin = c.d0; g.Cout = c.d1; g.stride = c.stride; g.pad = c.pad; g.K = c.K;
    g.ntaps = (c.K + c.stride - 1) / c.stride;
    g.N = c.stride * g.Cout; g.off0 = 0; g.offstep = -1; g.x3 = x3;
    g.w_off = reserve((size_t)g.ntaps * g.N * g.Cin * kmul() * esize());
    reserve_x3_second(g);
    add_jobs(kConvT, c.w.data(), g, g.Cin, c.K, c.stride);
    g.b_off = biases.size();
    for (int n = 0; n < g.Cout; ++n) biases.push_back(c.b.empty() ? 0.0f : c.b[n]);
    return g;
  }

  // BF16 arena: [tap][N][Cin] (K-major B operand); FP32: [tap][Cin][N].
  // src(n, ci) is the value of packed element (tap b.j, column n, channel ci).
  // Geometry is read into locals first: the stores could otherwise alias it.
  template <typename F>
  void fill(const Job& b, F src) {
    const int Cin = b.Cin, N = b.N, j = b.j, n0 = b.n0, n1 = b.n1;
    uint8_t* base = arena.get() + b.base;
    if (x3 && b.kind == kIdentity) {  // [I I I] against [X2 X1 X0]: a residual, exactly
      uint16_t* out = reinterpret_cast<uint16_t*>(base);
      for (int n = n0; n < n1; ++n) {
        uint16_t* row = out + ((size_t)j * N + n) * 3 * Cin;
        for (int k = 0; k < 3; ++k)
          for (int ci = 0; ci < Cin; ++ci)
            row[k * Cin + ci] = __bfloat16_as_ushort(__float2bfloat16_rn(n == ci ? 1.0f : 0.0f));
      }
      return;
    }
    if (x3) {
      // Row (tap j, column n) of the first block: [W0 W1 W2 W0 W1] (paired
      // with activation planes [X2 X1 X0 X1 X0]); of the second: W0.  W0..W2
      // are the three bf16 pieces of each weight.
      uint16_t* out = reinterpret_cast<uint16_t*>(base);
      uint16_t* out2 = reinterpret_cast<uint16_t*>(arena.get() + b.base2);
      for (int n = n0; n < n1; ++n) {
        uint16_t* row = out + ((size_t)j * N + n) * 5 * Cin;
        uint16_t* row2 = out2 + ((size_t)j * N + n) * Cin;
        for (int ci = 0; ci < Cin; ++ci) {
          float r = src(n, ci);
          uint16_t pc[3];
          for (int k = 0; k < 3; ++k) {
            const __nv_bfloat16 hb = __float2bfloat16_rn(r);
            pc[k] = __bfloat16_as_ushort(hb);
            r = r - __bfloat162float(hb);
          }
          const int piece[5] = {0, 1, 2, 0, 1};
          for (int k = 0; k < 5; ++k) row[k * Cin + ci] = pc[piece[k]];
          row2[ci] = pc[0];
        }
      }
      return;
    }
    if (dt == Dt::BF16) {
      uint16_t* out = reinterpret_cast<uint16_t*>(base);
      for (int n = n0; n < n1; ++n) {
        uint16_t* row = out + ((size_t)j * N + n) * Cin;
        for (int ci = 0; ci < Cin; ++ci) row[ci] = __bfloat16_as_ushort(__float2bfloat16_rn(src(n, ci)));
      }
    } else {
      // A transpose: 32-channel blocks keep both the reads (along ci) and the
      // writes (along n) in a few cache lines each.
      float* out = reinterpret_cast<float*>(base) + (size_t)j * Cin * N;
      for (int c0 = 0; c0 < Cin; c0 += 32) {
        const int c1 = std::min(Cin, c0 + 32);
        for (int n = n0; n < n1; ++n)
          for (int ci = c0; ci < c1; ++ci) out[(size_t)ci * N + n] = src(n, ci);
      }
    }
  }
  void run(const Job& b) {
    const int Cin = b.Cin, Cout = b.Cout, K = b.K, stride = b.stride, j = b.j;
    const float* w = b.w;
    switch (b.kind) {
      case kConv:
        if (b.rows) {
          const int* rows = b.rows;
          fill(b, [=](int n, int ci) { return w[((size_t)rows[n] * Cin + ci) * K + j]; });
        } else {
          fill(b, [=](int n, int ci) { return w[((size_t)n * Cin + ci) * K + j]; });
        }
        break;
      case kConvT:
        fill(b, [=](int n, int ci) {
          const int phi = n / Cout, o = n - phi * Cout, kk = phi + j * stride;
          return kk < K ? w[((size_t)ci * Cout + o) * K + kk] : 0.0f;
        });
        break;
      default:
        fill(b, [](int n, int ci) { return n == ci ? 1.0f : 0.0f; });
    }
  }
  void finish() {
    arena.reset(new uint8_t[std::max<size_t>(size, 1)]);
    for (const auto& gp : gaps) memset(arena.get() + gp.first, 0, gp.second);
    parallel_for(jobs.size(), [&](size_t i) { run(jobs[i]); });
    jobs.clear();
    owned.clear();
    owned_rows.clear();
  }
};

struct Stage {
  GemmConv up;
  std::vector<std::vector<GemmConv>> c1, c2;  // [branch][step]
};

}  // namespace
}  // namespace gsv

using namespace gsv;

struct gsvdec {
  int mode = GSV_MODE_FP32;
  int device = 0;
  Dt dt = Dt::F32;
  int in_ch = 0, C0 = 0, gin = 0, hop = 1;
  bool has_cond = false;
  GemmConv pre;
  std::vector<Stage> stages;
  // conv_post (one output channel): weights [K][C] fp32 on device
  int post_K = 0, post_pad = 0, post_C = 0;
  float post_bias = 0.0f;
  // device arenas
  void* d_w = nullptr;
  float* d_bias = nullptr;
  float* d_cond_w = nullptr;  // [C0][gin]
  float* d_cond_b = nullptr;
  float* d_post_w = nullptr;
  PostWeights post_wh{};  // the same [K][C] weights by value (K <= 16)
  bool post_wh_ok = false;
  // Error word of the bounded device waits: pinned, mapped host memory, so
  // the host can read what a stream-async call's kernels reported without a
  // copy or a sync (h_err), while the kernels write it through d_err.
  int* h_err = nullptr;
  int* d_err = nullptr;
  std::map<int, size_t> ident_off;  // bf16: identity weights per channel width
  // GSV_MODE_FP32_TC: the decoder's convs packed as three-piece K lists in a
  // second arena (same geometry and biases as pre / stages).
  bool x3 = false;
  GemmConv xpre;
  std::vector<Stage> xstages;
  void* d_wx = nullptr;
  size_t wx_bytes = 0;
  std::map<int, size_t> xident_off;  // three-piece identities [I I I] per channel width
  std::map<std::string, GemmConv> layers;  // every tap-GEMM conv by its dec.* prefix
  std::string layer_names;                 // newline-separated, in forward order
  void* lws = nullptr;                     // single-layer workspace
  size_t lws_bytes = 0;
  size_t w_bytes = 0;
  // workspace
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // FP32 mode: split-K partial sums of the forward in flight (inside ws)
  float* cur_part = nullptr;
  long long cur_part_cap = 0;
  // stage timing (level 1) and per-launch profile (level 2)
  int timing = 0;
  cudaEvent_t ev[32] = {};
  int n_ev = 0;
  float stage_ms[5] = {0, 0, 0, 0, 0};
  int launches = 0;
  struct Rec {
    std::string name;
    int kind, nconv;
    double flops, bytes;
    double cf[6], cb[6];
  };
  // Level 2 keeps one event list per forward until the stats are read, so a
  // timed loop of forwards needs no host sync: runs[k][0] starts forward k,
  // runs[k][i + 1] ends its launch i.
  std::vector<std::vector<cudaEvent_t>> runs;
  std::vector<std::vector<Rec>> run_recs;
  std::vector<cudaEvent_t> pool;
  std::vector<gsvdec_launch_stat> stats;
  // Flow inverse (present when the tensors include flow.flows.*).  Channels
  // are never moved for the flips: each layer's weights are packed against
  // the physical channel order that layer sees.
  struct FlowLayer {
    GemmConv pre;                  // 1x1, all C physical channels in (x1 weights zero) -> hid
    std::vector<GemmConv> in;      // WN in_layers, hid -> 2 hid, k taps
    std::vector<GemmConv> res;     // residual halves of res_skip 0 .. n-2, hid -> hid
    std::vector<GemmConv> post;    // coupling update, one segment per WN layer, hid -> C
    bool has_cond = false;
  };
  float* d_flow_cond_w = nullptr;  // every layer's cond_layer stacked: [layers * 2 hid n][gin]
  float* d_flow_cond_b = nullptr;
  bool flow_gate_fused = false;    // bf16: the WN gate runs in the in_layer GEMM's epilogue
  std::vector<FlowLayer> flow;
  int flow_C = 0, flow_half = 0, flow_hid = 0, flow_nwn = 0, flow_gin = 0;
  int* d_flow_perm = nullptr;      // physical channel of each output channel
  std::vector<int> flow_perm_host;
  void* fws = nullptr;
  size_t fws_bytes = 0;
  // EncP chains (present when the tensors include enc_p.* encoder layers).
  struct EncpLayer {
    GemmConv ffn1, ffn2;
    size_t norm = 0;  // float offset of gamma1, beta1, gamma2, beta2 (C each) in d_encp_norm
  };
  std::vector<EncpLayer> encp[3];
  GemmConv encp_proj;
  bool has_encp_proj = false;
  int encp_C = 0, encp_F = 0;
  float* d_encp_norm = nullptr;
  void* ews = nullptr;
  size_t ews_bytes = 0;
  // Multi-device decode (gsvdec_forward_multi): this handle's worker stream
  // and events, created on first use on the handle's device.
  cudaStream_t mstream = nullptr;
  cudaEvent_t mev_in = nullptr, mev_done = nullptr;
  // Overlapped host-memory forward (GSV_MEM_HOST_ASYNC): input copies, decode
  // and output copies on three streams, two staging slots used alternately so
  // one call's copies overlap the neighbouring calls' decodes.
  struct AsyncSlot {
    float* z = nullptr;
    float* g = nullptr;
    int* len = nullptr;
    float* wav = nullptr;
    cudaEvent_t in_done = nullptr, comp_done = nullptr, out_done = nullptr;
  };
  AsyncSlot aslot[2];
  cudaStream_t cs_in = nullptr, cs_comp = nullptr, cs_out = nullptr;
  cudaEvent_t ev_join = nullptr;
  void* aws = nullptr;  // both slots' staging
  size_t aws_bytes = 0;
  unsigned aseq = 0;
  bool async_run = false;  // the last call using the decoder workspace was an overlapped one
  cudaStream_t async_stream = nullptr;  // ... made with this stream
};

namespace gsv {
namespace {

size_t act_bytes(const gsvdec* h) { return h->dt == Dt::F32 ? 4 : 2; }
// Bytes per element of the decoder forward's activations (three bf16 pieces
// in GSV_MODE_FP32_TC).
size_t fwd_act_bytes(const gsvdec* h) { return h->x3 ? 6 : act_bytes(h); }
// Element type of the decoder forward's activations.
Dt fwd_dt(const gsvdec* h) { return h->x3 ? Dt::X3 : h->dt; }

// GEMM column col of a fused-gate in_layer holds original channel gate_src:
// column 32p + r is tanh-half channel 16p + r (r < 16), else sigmoid-half
// channel hid + 16p + (r - 16).
int gate_src(int col, int hid) {
  const int p = col / 32, r = col % 32;
  return r < 16 ? 16 * p + r : hid + 16 * p + (r - 16);
}

// Packs the flow for the inverse direction (ResidualCouplingBlock::forward
// with reverse = true, src/models/sovits_flow.rs:385-405).  With the
// activations time-major the channel flips (:408-414) become permutations of
// packed weight rows/columns: layer l sees the physical order pi_l (its
// logical channel j lives at physical pi_l[j]).  The coupling update of a
// mean-only layer, x1 <- x1 - mask * (post(mask * sum_j skip_j(acts_j)) +
// b_post) (:286-335, WN :155-167), is linear in the WN activations, so it is
// packed as ONE tap GEMM with a segment per WN layer, weights
// -W_post * W_skip_j (folded in double precision) and bias
// -(W_post * sum_j b_skip_j + b_post), placed on x1's physical rows; the
// residual x enters as an identity segment and x0 passes through unchanged.
int pack_flow(gsvdec* h, Packer& pk, const HostFlow& hf, std::vector<std::vector<float>>& cond_w,
              std::vector<std::vector<float>>& cond_b) {
  const HostCoupling& c0 = hf.layers[0];
  const int half = c0.pre.d1, hid = c0.pre.d0, C = 2 * half, nl = (int)c0.in.size();
  const int gin = c0.has_cond ? c0.cond.d1 : 0;
  for (const HostCoupling& c : hf.layers) {
    if (c.pre.d1 != half || c.pre.d0 != hid || c.pre.K != 1 || (int)c.in.size() != nl)
      return set_err(GSV_E_SHAPE, "%s: flow coupling layers differ in shape", c.pre.name.c_str());
    if (c.post.d1 != hid || c.post.K != 1)
      return set_err(GSV_E_SHAPE, "%s: post must be a 1x1 conv from %d channels", c.post.name.c_str(), hid);
    if (c.post.d0 != half)
      return set_err(GSV_E_UNSUPPORTED, "%s: only mean-only coupling layers (%d outputs) are supported, got %d",
                     c.post.name.c_str(), half, c.post.d0);
    for (int j = 0; j < nl; ++j) {
      if (c.in[j].d0 != 2 * hid || c.in[j].d1 != hid || c.in[j].K % 2 == 0)
        return set_err(GSV_E_SHAPE, "%s: expected [%d, %d, odd k]", c.in[j].name.c_str(), 2 * hid, hid);
      if (c.rs[j].d0 != (j < nl - 1 ? 2 * hid : hid) || c.rs[j].d1 != hid || c.rs[j].K != 1)
        return set_err(GSV_E_SHAPE, "%s: unexpected res/skip shape", c.rs[j].name.c_str());
    }
    if (c.has_cond != c0.has_cond || (c.has_cond && (c.cond.d0 != 2 * hid * nl || c.cond.K != 1 || c.cond.d1 != gin)))
      return set_err(GSV_E_SHAPE, "%s: cond_layer must be [%d, gin, 1] in every layer", c.pre.name.c_str(), 2 * hid * nl);
  }
  const int n = (int)hf.layers.size();
  h->flow.assign(n, {});
  h->flow_gate_fused = h->dt == Dt::BF16 && hid % 16 == 0;
  h->flow_C = C; h->flow_half = half; h->flow_hid = hid; h->flow_nwn = nl; h->flow_gin = gin;
  cond_w.assign(n, {});
  cond_b.assign(n, {});
  std::vector<int> pi(C);
  for (int j = 0; j < C; ++j) pi[j] = j;
  for (int l = n - 1; l >= 0; --l) {
    const HostCoupling& c = hf.layers[l];
    gsvdec::FlowLayer& F = h->flow[l];
    std::vector<int> q(C);
    for (int j = 0; j < C; ++j) q[j] = pi[C - 1 - j];  // flip
    pi = q;
    HostConv pre;
    pre.name = c.pre.name; pre.d0 = hid; pre.d1 = C; pre.K = 1; pre.pad = 0;
    pre.w.assign((size_t)hid * C, 0.0f);
    for (int o = 0; o < hid; ++o)
      for (int j = 0; j < half; ++j) pre.w[(size_t)o * C + pi[j]] = c.pre.w[(size_t)o * half + j];
    pre.b = c.pre.b;
    F.pre = pk.conv(std::move(pre));
    for (int j = 0; j < nl; ++j) {
      if (!h->flow_gate_fused) {
        F.in.push_back(pk.conv(c.in[j]));
        continue;
      }
      // Columns interleaved in 16-channel (tanh half, sigmoid half) pairs, so
      // one 32-column epilogue run holds both halves of 16 outputs.
      std::vector<int> rows(2 * hid);
      for (int col = 0; col < 2 * hid; ++col) rows[col] = gate_src(col, hid);
      F.in.push_back(pk.conv_rows(c.in[j], std::move(rows), 2 * hid));
    }
    for (int j = 0; j + 1 < nl; ++j) {
      // The residual half: the first hid rows of res_skip j (1x1, pad 0).
      F.res.push_back(pk.conv_rows(c.rs[j], {}, hid));
    }
    // Coupling update weights and bias (double precision fold).
    std::vector<double> cb(half, 0.0);
    for (int i = 0; i < half; ++i) cb[i] = c.post.b.empty() ? 0.0 : c.post.b[i];
    std::vector<std::vector<double>> wp(nl, std::vector<double>((size_t)half * hid, 0.0));
    // Rows i are independent (each sums over j, then k, in that order).
    parallel_for((size_t)half, [&](size_t ii) {
      const int i = (int)ii;
      for (int j = 0; j < nl; ++j) {
        const HostConv& rs = c.rs[j];
        const int r0 = j < nl - 1 ? hid : 0;  // skip rows of res_skip j
        double* dst = &wp[j][(size_t)i * hid];
        for (int k = 0; k < hid; ++k) {
          const double wpk = c.post.w[(size_t)i * hid + k];
          if (!rs.b.empty()) cb[i] += wpk * rs.b[r0 + k];
          const float* srow = &rs.w[(size_t)(r0 + k) * hid];
          for (int m = 0; m < hid; ++m) dst[m] += wpk * srow[m];
        }
      }
    });
    for (int j = 0; j < nl; ++j) {
      HostConv u;
      u.name = c.post.name; u.d0 = C; u.d1 = hid; u.K = 1; u.pad = 0;
      u.w.assign((size_t)C * hid, 0.0f);
      u.b.assign(C, 0.0f);
      for (int i = 0; i < half; ++i) {
        const int row = pi[half + i];
        for (int m = 0; m < hid; ++m) u.w[(size_t)row * hid + m] = (float)-wp[j][(size_t)i * hid + m];
        if (j == 0) u.b[row] = (float)-cb[i];
      }
      F.post.push_back(pk.conv(std::move(u)));
    }
    if (c.has_cond) {
      F.has_cond = true;
      // [2 hid n][gin][1]; with the fused gate each WN layer's 2 hid rows are
      // interleaved like its in_layer columns.
      cond_w[l].resize(c.cond.w.size());
      cond_b[l].assign(c.cond.d0, 0.0f);
      for (int r = 0; r < c.cond.d0; ++r) {
        const int j = r / (2 * hid), col = r % (2 * hid);
        const int src = j * 2 * hid + (h->flow_gate_fused ? gate_src(col, hid) : col);
        std::copy(c.cond.w.begin() + (size_t)src * gin, c.cond.w.begin() + (size_t)(src + 1) * gin,
                  cond_w[l].begin() + (size_t)r * gin);
        if (!c.cond.b.empty()) cond_b[l][r] = c.cond.b[src];
      }
    }
  }
  std::vector<int>& perm = pi;  // output channel j = physical pi[j]
  h->flow_perm_host = perm;
  if (h->dt == Dt::BF16) {
    if (!h->ident_off.count(C)) h->ident_off[C] = pk.identity(C);
    if (!h->ident_off.count(hid)) h->ident_off[hid] = pk.identity(hid);
  }
  return GSV_OK;
}

// Largest activation (elements per utterance) over all layers, for T0 frames.
size_t max_act_elems(const gsvdec* h, int T0) {
  size_t m = (size_t)T0 * std::max(h->C0, h->in_ch);
  int L = T0;
  for (const Stage& s : h->stages) {
    L = s.up.Lout(L);
    m = std::max(m, (size_t)L * s.up.Cout);
  }
  return m;
}

int out_len(const gsvdec* h, int T0) {
  int L = T0;
  for (const Stage& s : h->stages) L = s.up.Lout(L);
  return L;
}

struct Workspace {
  void* zin;
  void* buf[12];  // X, AX, OUT, XR0-2, AXR0-2, T0-2
  float* bias_bc;
  int* lens;
  float* zstage;  // host-mode staging of z / g / wav
  float* gstage;
  int* lstage;
  float* wav;
  float* tap;     // fp32 time-major tap scratch (debug taps only)
  float* part;    // FP32 mode: split-K partial sums of small launches (or null)
  long long part_cap;
};

// Split-K scratch of the FP32 CUDA-core kernel: small launches (batch 1,
// early stages) split their input-channel loop and reduce in order.
constexpr long long kSplitScratchFloats = 1LL << 24;  // 64 MB

int ensure_ws(gsvdec* h, int B, int T0, bool with_tap, Workspace& w, cudaStream_t drain = nullptr) {
  const size_t act = max_act_elems(h, T0) * (size_t)B;
  const size_t eb = fwd_act_bytes(h);
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const int L = out_len(h, T0);
  size_t need = 0;
  size_t o_zin = need; need += al((size_t)B * T0 * h->in_ch * eb);
  size_t o_buf = need; need += 12 * al(act * eb);
  size_t o_bbc = need; need += al((size_t)B * h->C0 * 4);
  size_t o_len = need; need += al((size_t)B * 16 * 4);
  size_t o_zs = need; need += al((size_t)B * T0 * h->in_ch * 4);
  size_t o_gs = need; need += al((size_t)B * std::max(h->gin, 1) * 4);
  size_t o_ls = need; need += al((size_t)B * 4);
  size_t o_wav = need; need += al((size_t)B * L * 4);
  size_t o_tap = need; if (with_tap) need += al(act * 4);
  const size_t part_floats = h->dt == Dt::F32 ? (size_t)kSplitScratchFloats : 0;
  size_t o_part = need; need += al(part_floats * 4);
  if (need > h->ws_bytes) {
    if (drain) CUDA_TRY(cudaStreamSynchronize(drain));  // work in flight there may still use it
    if (h->ws) CUDA_TRY(cudaFree(h->ws));
    h->ws = nullptr;
    h->ws_bytes = 0;
    CUDA_TRY(dev_malloc(&h->ws, need));
    h->ws_bytes = need;
  }
  char* p = static_cast<char*>(h->ws);
  w.zin = p + o_zin;
  for (int i = 0; i < 12; ++i) w.buf[i] = p + o_buf + i * al(act * eb);
  w.bias_bc = reinterpret_cast<float*>(p + o_bbc);
  w.lens = reinterpret_cast<int*>(p + o_len);
  w.zstage = reinterpret_cast<float*>(p + o_zs);
  w.gstage = reinterpret_cast<float*>(p + o_gs);
  w.lstage = reinterpret_cast<int*>(p + o_ls);
  w.wav = reinterpret_cast<float*>(p + o_wav);
  w.tap = with_tap ? reinterpret_cast<float*>(p + o_tap) : nullptr;
  w.part = part_floats ? reinterpret_cast<float*>(p + o_part) : nullptr;
  w.part_cap = (long long)part_floats;
  return GSV_OK;
}

// part (three-piece convs only): 0 = the five small-product blocks, 1 = the
// large-product block.
TapSeg make_seg(const gsvdec* h, const GemmConv& g, const void* x, int Lin, int part = 0) {
  TapSeg s{};
  s.x = x;
  s.w = static_cast<const char*>(g.x3 ? h->d_wx : h->d_w) + (part ? g.w_off2 : g.w_off);
  s.Lin = Lin;
  s.Cin = g.x3 && !part ? 5 * g.Cin : g.Cin;
  s.pc = g.x3 ? g.Cin : 0;
  s.ntaps = g.ntaps;
  s.off0 = g.off0;
  s.offstep = g.offstep;
  return s;
}

TapConv make_op(const gsvdec* h, const GemmConv& g, int B, const void* x, int Lin) {
  TapConv op{};
  op.seg[0] = make_seg(h, g, x, Lin);
  op.nseg = 1;
  if (g.x3) {  // small products first, the large one last (fewer roundings against the big sum)
    op.seg[1] = make_seg(h, g, x, Lin, 1);
    op.nseg = 2;
  }
  op.B = B;
  op.Q = g.Q(Lin);
  op.N = g.N;
  op.Cout = g.Cout;
  op.Lout = g.Lout(Lin);
  op.crop = g.transposed ? g.pad * g.Cout : 0;
  op.bias = h->d_bias + g.b_off;
  op.div = 1.0f;
  op.slope = 0.1f;
  op.split = g.x3 ? 1 : 0;
  return op;
}

// Records the end of one kernel launch (per-launch profile, timing level 2).
int after_launch(gsvdec* h, cudaStream_t st, const std::string& name, int kind, int nconv,
                 double flops, double bytes, const double* cf = nullptr,
                 const double* cb = nullptr) {
  h->launches++;
  if (h->timing < 2 || h->runs.empty()) return GSV_OK;
  cudaEvent_t e;
  if (!h->pool.empty()) {
    e = h->pool.back();
    h->pool.pop_back();
  } else {
    CUDA_TRY(cudaEventCreate(&e));
  }
  CUDA_TRY(cudaEventRecord(e, st));
  h->runs.back().push_back(e);
  gsvdec::Rec rec{name, kind, nconv, flops, bytes, {0, 0, 0, 0, 0, 0}, {0, 0, 0, 0, 0, 0}};
  for (int i = 0; i < 6 && i < nconv; ++i) {
    rec.cf[i] = cf ? cf[i] : (i == 0 ? flops : 0.0);
    rec.cb[i] = cb ? cb[i] : (i == 0 ? bytes : 0.0);
  }
  h->run_recs.back().push_back(rec);
  return GSV_OK;
}

// Algorithmic work of one reference conv inside a tap GEMM (see gsvdec.h).
struct Work {
  double flops = 0, bytes = 0;
  double cf[6] = {0, 0, 0, 0, 0, 0}, cb[6] = {0, 0, 0, 0, 0, 0};
  int nconv = 0;
  void add(const GemmConv& g, int B, int Lin, int nres, double e) {
    const int Lout = g.Lout(Lin);
    const double f = 2.0 * g.Cin * g.Cout * g.K * (double)Lin * B;
    const double by = e * B * ((double)g.Cin * Lin + (double)g.Cout * Lout) +
                      e * (double)g.Cin * g.Cout * g.K + e * B * (double)g.Cout * Lout * nres;
    if (nconv < 6) { cf[nconv] = f; cb[nconv] = by; }
    flops += f;
    bytes += by;
    nconv++;
  }
  // A reference conv Cin -> Cout, k taps, over L frames (unfused layer I/O).
  void add_ref(int Cin, int Cout, int k, int L, int B, double e) {
    const double f = 2.0 * Cin * Cout * k * (double)L * B;
    const double by = e * B * ((double)Cin + Cout) * L + e * (double)Cin * Cout * k;
    if (nconv < 6) { cf[nconv] = f; cb[nconv] = by; }
    flops += f;
    bytes += by;
    nconv++;
  }
};

constexpr int kIdentityResidualMinC = 32;

int run_group(gsvdec* h, TapConvGroup& grp, cudaStream_t st, const std::string& name,
              const Work& wk) {
  grp.err = h->d_err;
  grp.partial = h->cur_part;
  grp.partial_cap = h->cur_part_cap;
  cudaError_t e;
  if (grp.op[0].split) {
    // Three-piece ops (GSV_MODE_FP32_TC): a single residual enters the GEMM as
    // a last segment [X2 X1 X0] against [I I I] (after the large products:
    // three more roundings of the sum); the three-residual branch sums add
    // theirs in the epilogue in fp32, each read as the sum of its pieces.
    for (int i = 0; i < grp.n; ++i) {
      TapConv& op = grp.op[i];
      if (!op.split) return set_err(GSV_E_UNSUPPORTED, "%s mixes three-piece and plain ops", name.c_str());
      if (op.nres != 1) continue;
      auto it = h->xident_off.find(op.Cout);
      if (it == h->xident_off.end() || op.N != op.Cout || op.crop != 0 || op.Q != op.Lout || op.nseg >= kMaxSeg)
        return set_err(GSV_E_UNSUPPORTED, "residual of %s cannot be folded into the GEMM", name.c_str());
      TapSeg& sg = op.seg[op.nseg++];
      sg = TapSeg{};
      sg.x = op.res[0];
      sg.w = static_cast<const char*>(h->d_wx) + it->second;
      sg.Lin = op.Lout;
      sg.Cin = 3 * op.Cout;
      sg.pc = op.Cout;
      sg.ntaps = 1;
      sg.off0 = 0;
      sg.offstep = 1;
      op.nres = 0;
    }
    bool tc = true;
    for (int i = 0; i < grp.n; ++i) tc = tc && tapconv_tc_supported(grp.op[i]);
    if (!tc) return set_err(GSV_E_UNSUPPORTED, "layer geometry not supported by the tcgen05 kernel");
    if (grp.op[0].Cout <= 32 && grp.n > 1) {
      // Narrow three-piece ops keep their weights resident in shared memory
      // (six K blocks per tap): one launch per op, so one op's weights fit.
      e = cudaSuccess;
      for (int i = 0; i < grp.n && e == cudaSuccess; ++i) {
        TapConvGroup one{};
        one.op[0] = grp.op[i];
        one.n = 1;
        one.err = grp.err;
        e = launch_tapconv_tc(one, st);
      }
      h->launches += grp.n - 1;
    } else {
      e = launch_tapconv_tc(grp, st);
    }
  } else if (h->dt == Dt::F32) {
    e = launch_tapconv_f32(grp, st);
  } else {
    // Residuals of wide layers enter the tensor-core GEMM as identity-weight
    // segments (no global loads in the epilogue); narrow layers read them in
    // the epilogue instead (an extra TMA window costs more there than the MMA
    // saves), and so do convs whose input width differs from Cout (every GEMM
    // segment shares one input width).  The three-residual branch sums at
    // >= 128 channels also read theirs in the epilogue (256-bit loads): three
    // identity segments there cost 24 MMAs per tile on top of 168 (rb1's
    // branch sum 0.448 -> 0.416 ms on B200; single-residual conv2 and the
    // narrower sums measured slower that way).
    for (int i = 0; i < grp.n; ++i) {
      TapConv& op = grp.op[i];
      if (op.nres == 0 || op.Cout < kIdentityResidualMinC || op.seg[0].Cin != op.Cout) continue;
      if (op.nres >= 2 && op.Cout >= 128) continue;
      auto it = h->ident_off.find(op.Cout);
      if (it == h->ident_off.end() || op.N != op.Cout || op.crop != 0 || op.Q != op.Lout ||
          op.nseg + op.nres > kMaxSeg)
        return set_err(GSV_E_UNSUPPORTED, "residual of %s cannot be folded into the GEMM", name.c_str());
      for (int r = 0; r < op.nres; ++r) {
        TapSeg& sg = op.seg[op.nseg++];
        sg.x = op.res[r];
        sg.w = static_cast<const char*>(h->d_w) + it->second;
        sg.Lin = op.Lout;
        sg.Cin = op.Cout;
        sg.ntaps = 1;
        sg.off0 = 0;
        sg.offstep = 1;
      }
      op.nres = 0;
    }
    bool tc = true;
    for (int i = 0; i < grp.n; ++i) tc = tc && tapconv_tc_supported(grp.op[i]);
    e = tc ? launch_tapconv_tc(grp, st) : cudaErrorNotSupported;
    if (!tc) return set_err(GSV_E_UNSUPPORTED, "layer geometry not supported by the tcgen05 kernel");
  }
  if (e != cudaSuccess) return set_err(GSV_E_CUDA, "tap-conv launch failed: %s", cudaGetErrorString(e));
  return after_launch(h, st, name, 0, wk.nconv, wk.flops, wk.bytes, wk.cf, wk.cb);
}

int run_one(gsvdec* h, const TapConv& op, cudaStream_t st, const std::string& name,
            const Work& wk) {
  TapConvGroup g{};
  g.op[0] = op;
  g.n = 1;
  return run_group(h, g, st, name, wk);
}

void mark(gsvdec* h, cudaStream_t st) {
  if (h->timing == 1 && h->n_ev < 32) cudaEventRecord(h->ev[h->n_ev++], st);
}

// The whole forward on device buffers.  zsrc is NCL fp32 [B][in_ch][Tsrc]
// (frames t_off .. t_off+T0), gdev [B][gin] or null, lens_in [B] or null.
// taps (host, optional): reference-layout copies of each stage.
// Decodes of at most this many frames (B x T0) launch with programmatic
// dependent launch: their launches are short and sub-wave, so the next
// kernel's set-up overlapping the tail of the one before pays.  Measured on
// B200 (bf16, same build with and without): one utterance of 407 / 782 /
// 1532 / 3000 frames 0.99 -> 0.87, 1.42 -> 1.32, 2.23 -> 2.17, 3.93 -> 3.90 ms;
// the 16 x 500 batch 10.17 -> 10.33 ms (slower), so it stays off there.
constexpr int64_t kPdlDecodeMaxFrames = 4096;

int forward_device(gsvdec* h, const float* zsrc, int Tsrc, int t_off, const float* gdev,
                   const int* lens_in, int B, int T0, float* wav_dev, Workspace& w,
                   float* const* taps, cudaStream_t st) {
  PdlScope pdl((int64_t)B * T0 <= kPdlDecodeMaxFrames);
  // This forward's split-K scratch (FP32 mode), for run_group, until it returns.
  struct PartScope {
    gsvdec* h;
    PartScope(gsvdec* hh, float* p, long long cap) : h(hh) {
      h->cur_part = p;
      h->cur_part_cap = p ? cap : 0;
    }
    ~PartScope() {
      h->cur_part = nullptr;
      h->cur_part_cap = 0;
    }
  } part_scope(h, w.part, w.part_cap);
  h->launches = 0;
  h->n_ev = 0;
  if (h->timing >= 2) {
    cudaEvent_t e;
    if (!h->pool.empty()) {
      e = h->pool.back();
      h->pool.pop_back();
    } else {
      CUDA_TRY(cudaEventCreate(&e));
    }
    CUDA_TRY(cudaEventRecord(e, st));
    h->runs.push_back({e});
    h->run_recs.push_back({});
  }
  mark(h, st);
  const double eb = (double)act_bytes(h);
  void* X = w.buf[0];
  void* AX = w.buf[1];
  void* OUT = w.buf[2];
  void* XR[3] = {w.buf[3], w.buf[4], w.buf[5]};
  void* AXR[3] = {w.buf[6], w.buf[7], w.buf[8]};
  void* TT[3] = {w.buf[9], w.buf[10], w.buf[11]};
  const int nst = (int)h->stages.size();
  // Per-stage valid lengths (only when masking).
  const int* lens = nullptr;
  if (lens_in) {
    int mul[16], add[16];
    if (nst > 15) return set_err(GSV_E_UNSUPPORTED, "more than 15 upsample stages");
    for (int s = 0; s < nst; ++s) {
      const GemmConv& u = h->stages[s].up;
      mul[s] = u.stride;
      add[s] = u.K - 2 * u.pad - u.stride;
    }
    CUDA_TRY(launch_lengths(lens_in, B, T0, mul, add, nst, w.lens, st));
    GSV_TRY(after_launch(h, st, "lengths", 1, 0, 0.0, 8.0 * B * (nst + 1)));
    lens = w.lens;
  }
  auto stage_len = [&](int s) -> const int* { return lens ? lens + (size_t)s * B : nullptr; };

  CUDA_TRY(launch_transpose_in(zsrc, B, h->in_ch, Tsrc, t_off, T0, lens ? lens : nullptr, w.zin, fwd_dt(h), st));
  GSV_TRY(after_launch(h, st, "input_relayout", 1, 0, 0.0, (4.0 + eb) * B * h->in_ch * T0));
  const float* bias_bc = nullptr;
  if (h->has_cond && gdev) {
    CUDA_TRY(launch_cond(gdev, h->d_cond_w, h->d_cond_b, B, h->gin, h->C0, w.bias_bc, st));
    GSV_TRY(after_launch(h, st, "cond", 1, 1, 2.0 * B * h->gin * h->C0,
                         4.0 * ((double)B * h->gin + (double)h->gin * h->C0 + (double)B * h->C0)));
    bias_bc = w.bias_bc;
  }
  auto tap_out = [&](int idx, const void* src, int L, int C) -> int {
    if (!taps || !taps[idx]) return GSV_OK;
    CUDA_TRY(launch_to_ncl(src, fwd_dt(h), B, L, C, w.tap, st));
    CUDA_TRY(cudaMemcpyAsync(taps[idx], w.tap, sizeof(float) * (size_t)B * L * C, cudaMemcpyDeviceToHost, st));
    return GSV_OK;
  };
  // conv_pre (+ cond, folded into a per-utterance bias), LeakyReLU for the
  // first upsample (:390-408).
  int L = T0;
  {
    TapConv op = make_op(h, h->x3 ? h->xpre : h->pre, B, w.zin, L);
    op.bias_bc = bias_bc;
    op.len = stage_len(0);
    op.out_act = OUT;
    op.slope = nst > 0 ? 0.1f : 0.01f;
    if (taps && taps[0]) op.out_raw = X;
    Work wk;
    wk.add(h->pre, B, L, 0, eb);
    GSV_TRY(run_one(h, op, st, "conv_pre", wk));
    GSV_TRY(tap_out(0, X, L, h->C0));
  }
  mark(h, st);
  for (int i = 0; i < nst; ++i) {
    const Stage& sg = (h->x3 ? h->xstages : h->stages)[i];
    const bool last = i + 1 == nst;
    const float next_slope = last ? 0.01f : 0.1f;
    const int nb = (int)sg.c1.size();
    const int Lin = L;
    L = sg.up.Lout(Lin);
    const int C = sg.up.Cout;
    const int* len = stage_len(i + 1);
    // Narrow stages in BF16 mode: ResBlock steps 0 and 1 run as fused
    // conv1 -> conv2 kernels (rbstep_tc.cu); the intermediate stays on chip.
    bool fuse = h->dt == Dt::BF16 && nb == 3 && rbstep_supported(C, 1, 1) && h->ident_off.count(C);
    for (int r = 0; r < nb && fuse; ++r) {
      fuse = sg.c1[r].size() == 3;
      for (int j = 0; j < 2 && fuse; ++j)
        fuse = rbstep_supported(C, sg.c1[r][j].ntaps, sg.c1[r][j].offstep) && sg.c1[r][j].off0 == -sg.c1[r][j].pad;
    }
    {
      TapConv op = make_op(h, sg.up, B, OUT, Lin);
      op.len = len;
      op.out_raw = X;
      // The fused step applies the LeakyReLU to its own input window, so the
      // upsample's activated copy is only needed by the unfused step 0.
      op.out_act = nb > 0 && !fuse ? AX : nullptr;
      if (nb == 0) { op.out_act = AX; op.slope = next_slope; }
      Work wk;
      wk.add(sg.up, B, Lin, 0, eb);
      GSV_TRY(run_one(h, op, st, "ups" + std::to_string(i), wk));
    }
    GSV_TRY(tap_out(1 + 2 * i, X, L, C));
    mark(h, st);
    if (nb == 0) {
      std::swap(OUT, AX);
      mark(h, st);
      continue;
    }
    int first_step = 0;
    if (fuse) {
      for (int j = 0; j < 2; ++j) {
        RbStepGroup rg{};
        rg.n = nb;
        rg.C = C;
        rg.B = B;
        rg.L = L;
        rg.len = len;
        rg.slope = 0.1f;
        rg.identity = static_cast<const char*>(h->d_w) + h->ident_off[C];
        rg.err = h->d_err;
        Work wk;
        for (int r = 0; r < nb; ++r) {
          const GemmConv& a = sg.c1[r][j];
          const GemmConv& c = sg.c2[r][j];
          RbStepOp& o = rg.op[r];
          o.x = j == 0 ? X : XR[r];
          o.w1 = static_cast<const char*>(h->d_w) + a.w_off;
          o.w2 = static_cast<const char*>(h->d_w) + c.w_off;
          o.b1 = h->d_bias + a.b_off;
          o.b2 = h->d_bias + c.b_off;
          o.out_raw = j == 0 ? XR[r] : TT[r];
          o.out_act = j == 0 ? nullptr : AXR[r];
          o.k = a.ntaps;
          o.d = a.offstep;
          wk.add(a, B, L, 0, eb);
          wk.add(c, B, L, 1, eb);
        }
        const cudaError_t e = launch_rbstep(rg, st);
        if (e != cudaSuccess) return set_err(GSV_E_CUDA, "fused resblock step launch failed: %s", cudaGetErrorString(e));
        h->launches += rg.n - 1;  // one kernel per branch
        GSV_TRY(after_launch(h, st, "rb" + std::to_string(i) + ".step" + std::to_string(j) + ".fused", 0,
                             wk.nconv, wk.flops, wk.bytes, wk.cf, wk.cb));
      }
      // Step 2: conv1 into XR (free now) from AXR, then the fused final op reads
      // t = XR and the raw step-1 output TT.
      std::swap(XR, TT);  // XR[r] now names the step-1 raw output; TT[r] the free buffers
      first_step = 2;
    }
    int max_steps = 0;
    for (int r = 0; r < nb; ++r) max_steps = std::max(max_steps, (int)sg.c1[r].size());
    for (int j = first_step; j < max_steps; ++j) {
      TapConvGroup g1{}, g2{};
      Work w1, w2;
      for (int r = 0; r < nb; ++r) {
        const int S = (int)sg.c1[r].size();
        if (j >= S) continue;
        TapConv a = make_op(h, sg.c1[r][j], B, j == 0 ? AX : AXR[r], L);
        a.len = len;
        a.out_act = TT[r];
        g1.op[g1.n++] = a;
        w1.add(sg.c1[r][j], B, L, 0, eb);
        if (j < S - 1) {
          TapConv c = make_op(h, sg.c2[r][j], B, TT[r], L);
          c.len = len;
          c.res[0] = j == 0 ? X : XR[r];
          c.nres = 1;
          c.out_raw = XR[r];
          c.out_act = AXR[r];
          g2.op[g2.n++] = c;
          w2.add(sg.c2[r][j], B, L, 1, eb);
        }
      }
      const std::string nm = "rb" + std::to_string(i) + ".step" + std::to_string(j);
      if (g1.n) GSV_TRY(run_group(h, g1, st, nm + ".conv1", w1));
      if (g2.n) GSV_TRY(run_group(h, g2, st, nm + ".conv2", w2));
    }
    // Last step of every branch in one op: the branch sum and the true
    // division by the branch count (:418-442) plus the next LeakyReLU.
    {
      TapConv f{};
      Work wf;
      for (int r = 0; r < nb; ++r) {
        const int S = (int)sg.c1[r].size();
        const GemmConv& g = sg.c2[r][S - 1];
        wf.add(g, B, L, 1, eb);
        if (r == 0) f = make_op(h, g, B, TT[r], L);
        else f.seg[r] = make_seg(h, g, TT[r], L);
        f.res[r] = S == 1 ? X : XR[r];
      }
      f.nseg = nb;
      if (h->x3) {  // every branch's small-product blocks first, then the large ones
        for (int r = 0; r < nb; ++r) {
          const GemmConv& g = sg.c2[r][sg.c2[r].size() - 1];
          f.seg[r] = make_seg(h, g, TT[r], L, 0);
          f.seg[nb + r] = make_seg(h, g, TT[r], L, 1);
        }
        f.nseg = 2 * nb;
      }
      f.nres = nb;
      f.bias = h->d_bias + sg.c2[0][sg.c2[0].size() - 1].b_off;  // replaced below when nb > 1
      f.div = (float)nb;
      f.len = len;
      f.out_act = OUT;
      f.slope = next_slope;
      if (taps && taps[2 + 2 * i]) f.out_raw = AX;  // AX is dead by now
      if (nb > 1) {
        // Summed bias of the branches' last convs lives right after the stage's
        // packed biases (set up at create time).
        f.bias = h->d_bias + sg.c2.back().back().b_off + sg.c2.back().back().Cout;
      }
      GSV_TRY(run_one(h, f, st, "rb" + std::to_string(i) + ".final", wf));
      GSV_TRY(tap_out(2 + 2 * i, AX, L, C));
    }
    mark(h, st);
  }
  // LeakyReLU(0.01) was applied by the producer; conv_post + tanh (:449-455).
  CUDA_TRY(launch_post(OUT, fwd_dt(h), B, L, h->post_C, h->d_post_w, h->post_wh_ok ? &h->post_wh : nullptr,
                       h->post_K, h->post_pad,
                       h->post_bias, stage_len(nst), wav_dev, taps && taps[1 + 2 * nst] ? w.tap : nullptr, st));
  GSV_TRY(after_launch(h, st, "conv_post", 2, 1, 2.0 * h->post_C * h->post_K * (double)L * B,
                       eb * B * (double)h->post_C * L + 4.0 * B * (double)L + 4.0 * h->post_C * h->post_K));
  if (taps && taps[1 + 2 * nst])
    CUDA_TRY(cudaMemcpyAsync(taps[1 + 2 * nst], w.tap, sizeof(float) * (size_t)B * L, cudaMemcpyDeviceToHost, st));
  mark(h, st);
  return GSV_OK;
}

// ---------------------------------------------------------------------------
// Flow inverse on device buffers.

struct FlowWs {
  void* x[2];      // [B][T][C] activations (ping-pong: the coupling update is not in place)
  void* hb[2];     // [B][T][hid] WN residual stream (ping-pong)
  void* xin;       // [B][T][2 hid] in_layer output
  void* act[16];   // [B][T][hid] gated activations, one per WN layer
  float* cond;     // [B][layers * 2 hid n] per-utterance cond projections of every coupling layer
  int* lens;       // [B] valid frames
  float* zstage;   // host-mode staging of z_p / g / lengths and of z
  float* gstage;
  int* lstage;
  float* zout;     // [B][C][T] fp32
};

int ensure_flow_ws(gsvdec* h, int B, int T0, FlowWs& w) {
  const size_t eb = act_bytes(h);
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t C = h->flow_C, hid = h->flow_hid, nl = h->flow_nwn;
  const size_t bt = (size_t)B * T0;
  size_t need = 0;
  size_t o_x = need; need += 2 * al(bt * C * eb);
  size_t o_h = need; need += 2 * al(bt * hid * eb);
  size_t o_xin = need; need += al(bt * 2 * hid * eb);
  size_t o_act = need; need += nl * al(bt * hid * eb);
  size_t o_cond = need; need += al((size_t)B * 2 * hid * nl * h->flow.size() * 4);
  size_t o_len = need; need += al((size_t)B * 4);
  size_t o_zs = need; need += al(bt * C * 4);
  size_t o_gs = need; need += al((size_t)B * std::max(h->flow_gin, 1) * 4);
  size_t o_ls = need; need += al((size_t)B * 4);
  size_t o_zo = need; need += al(bt * C * 4);
  if (need > h->fws_bytes) {
    if (h->fws) CUDA_TRY(cudaFree(h->fws));
    h->fws = nullptr;
    h->fws_bytes = 0;
    CUDA_TRY(dev_malloc(&h->fws, need));
    h->fws_bytes = need;
  }
  char* p = static_cast<char*>(h->fws);
  for (int i = 0; i < 2; ++i) {
    w.x[i] = p + o_x + i * al(bt * C * eb);
    w.hb[i] = p + o_h + i * al(bt * hid * eb);
  }
  w.xin = p + o_xin;
  for (size_t j = 0; j < nl && j < 16; ++j) w.act[j] = p + o_act + j * al(bt * hid * eb);
  w.cond = reinterpret_cast<float*>(p + o_cond);
  w.lens = reinterpret_cast<int*>(p + o_len);
  w.zstage = reinterpret_cast<float*>(p + o_zs);
  w.gstage = reinterpret_cast<float*>(p + o_gs);
  w.lstage = reinterpret_cast<int*>(p + o_ls);
  w.zout = reinterpret_cast<float*>(p + o_zo);
  return GSV_OK;
}

void begin_run(gsvdec* h, cudaStream_t st) {
  h->launches = 0;
  h->n_ev = 0;
  if (h->timing >= 2) {
    cudaEvent_t e;
    if (!h->pool.empty()) {
      e = h->pool.back();
      h->pool.pop_back();
    } else if (cudaEventCreate(&e) != cudaSuccess) {
      return;
    }
    cudaEventRecord(e, st);
    h->runs.push_back({e});
    h->run_recs.push_back({});
  }
}

// z = flow^-1(z_p) * y_mask (src/models/sovits_flow.rs:385-405 with reverse =
// true, then src/models/sovits.rs:394).  zp [B][C][T0] fp32, gdev [B][gin] or
// null, lens_in [B] or null, z_dev [B][C][T0] fp32.
int flow_device(gsvdec* h, const float* zp, const float* gdev, const int* lens_in, int B, int T0,
                float* z_dev, FlowWs& w, cudaStream_t st) {
  // Programmatic dependent launch for the flow's chain of short launches.
  PdlScope pdl(true);
  begin_run(h, st);
  const double eb = (double)act_bytes(h);
  const int C = h->flow_C, hid = h->flow_hid, nl = h->flow_nwn;
  const int* lens = nullptr;
  if (lens_in) {
    CUDA_TRY(launch_lengths(lens_in, B, T0, nullptr, nullptr, 0, w.lens, st));
    GSV_TRY(after_launch(h, st, "flow.lengths", 1, 0, 0.0, 8.0 * B));
    lens = w.lens;
  }
  CUDA_TRY(launch_transpose_in(zp, B, C, T0, 0, T0, lens, w.x[0], h->dt, st));
  GSV_TRY(after_launch(h, st, "flow.input_relayout", 1, 0, 0.0, (4.0 + eb) * B * C * T0));
  int cur = 0;
  const int n = (int)h->flow.size();
  const int cond_ld = 2 * hid * nl * n;  // every layer's projection in one row per utterance
  const bool cond = h->d_flow_cond_w && gdev;
  if (cond) {
    CUDA_TRY(launch_cond(gdev, h->d_flow_cond_w, h->d_flow_cond_b, B, h->flow_gin, cond_ld, w.cond, st));
    GSV_TRY(after_launch(h, st, "flow.cond", 1, 1, 2.0 * B * h->flow_gin * cond_ld,
                         4.0 * ((double)B * h->flow_gin + (double)h->flow_gin * cond_ld)));
  }
  for (int l = n - 1; l >= 0; --l) {
    const gsvdec::FlowLayer& F = h->flow[l];
    const std::string nm = "flow." + std::to_string(l);
    const int coff = l * 2 * hid * nl;
    {
      TapConv op = make_op(h, F.pre, B, w.x[cur], T0);
      op.len = lens;
      op.out_raw = w.hb[0];
      Work wk;
      wk.add_ref(h->flow_half, hid, 1, T0, B, eb);  // pre reads x0 only
      GSV_TRY(run_one(h, op, st, nm + ".pre", wk));
    }
    int hc = 0;
    for (int j = 0; j < nl; ++j) {
      {
        TapConv op = make_op(h, F.in[j], B, w.hb[hc], T0);
        op.len = lens;
        Work wk;
        wk.add(F.in[j], B, T0, 0, eb);
        if (h->flow_gate_fused) {
          // in_layer + cond + tanh * sigmoid in one launch (gated epilogue).
          op.gate = 1;
          op.out_raw = w.act[j];
          op.bias_bc = cond ? w.cond + coff + j * 2 * hid : nullptr;
          op.bias_bc_ld = cond_ld;
          GSV_TRY(run_one(h, op, st, nm + ".in" + std::to_string(j) + "+gate", wk));
        } else {
          op.out_raw = w.xin;
          GSV_TRY(run_one(h, op, st, nm + ".in" + std::to_string(j), wk));
          CUDA_TRY(launch_gate(w.xin, cond ? w.cond : nullptr, cond_ld, coff + j * 2 * hid, B, T0, hid, lens,
                               w.act[j], h->dt, st));
          GSV_TRY(after_launch(h, st, nm + ".gate" + std::to_string(j), 1, 0, 0.0, 3.0 * eb * B * hid * T0));
        }
      }
      if (j + 1 < nl) {
        TapConv op = make_op(h, F.res[j], B, w.act[j], T0);
        op.len = lens;
        op.res[0] = w.hb[hc];
        op.nres = 1;
        op.out_raw = w.hb[hc ^ 1];
        Work wk;
        wk.add_ref(hid, 2 * hid, 1, T0, B, eb);  // res_skip j (its skip half is folded into the update)
        GSV_TRY(run_one(h, op, st, nm + ".res" + std::to_string(j), wk));
        hc ^= 1;
      }
    }
    {
      TapConv op = make_op(h, F.post[0], B, w.act[0], T0);
      for (int j = 1; j < nl; ++j) op.seg[j] = make_seg(h, F.post[j], w.act[j], T0);
      op.nseg = nl;
      op.len = lens;
      op.res[0] = w.x[cur];
      op.nres = 1;
      op.out_raw = w.x[cur ^ 1];
      Work wk;
      wk.add_ref(hid, hid, 1, T0, B, eb);                 // the last res_skip (skip only)
      wk.add_ref(hid, h->flow_half, 1, T0, B, eb);        // post
      GSV_TRY(run_one(h, op, st, nm + ".couple", wk));
      cur ^= 1;
    }
  }
  CUDA_TRY(launch_to_ncl(w.x[cur], h->dt, B, T0, C, z_dev, st, h->d_flow_perm));
  GSV_TRY(after_launch(h, st, "flow.output_relayout", 1, 0, 0.0, (4.0 + eb) * B * C * T0));
  return GSV_OK;
}

// A kernel whose bounded wait gave up leaves a non-zero word in d_err.
// Called after the stream of the call has been synchronised: every kernel of
// this call (and of earlier stream-async calls on the same handle) has
// finished, so the word holds everything they reported.
int check_device_error(gsvdec* h) {
  volatile int* w = h->h_err;
  const int v = *w;
  if (v != 0) {
    *w = 0;
    return set_err(GSV_E_TIMEOUT,
                   "a device wait of this call or of an earlier stream-async call on this handle gave up "
                   "(code %d); its results are invalid", v);
  }
  return GSV_OK;
}

// Entry check of every call: a stream-async call returns before its kernels
// run, so a wait that gave up in one of them is reported here, by the next
// call on the handle, which then does nothing else (the word is cleared, so
// the call after it proceeds).  Reads host memory only: no sync.
int take_async_error(gsvdec* h) {
  volatile int* w = h->h_err;
  const int v = *w;
  if (v != 0) {
    *w = 0;
    return set_err(GSV_E_TIMEOUT,
                   "a device wait of an earlier stream-async call on this handle gave up (code %d); "
                   "that call's results are invalid (this call did not run)", v);
  }
  return GSV_OK;
}

int collect_timing(gsvdec* h, cudaStream_t st) {
  if (h->timing != 1 || h->n_ev < 3) return GSV_OK;
  CUDA_TRY(cudaStreamSynchronize(st));
  // events: [start, after pre, (after up_i, after rb_i) x nst, after post]
  float pre = 0, up = 0, rb = 0, post = 0, tot = 0;
  cudaEventElapsedTime(&pre, h->ev[0], h->ev[1]);
  int k = 1;
  for (size_t i = 0; i < h->stages.size() && k + 2 < h->n_ev; ++i) {
    float a = 0, b = 0;
    cudaEventElapsedTime(&a, h->ev[k], h->ev[k + 1]);
    cudaEventElapsedTime(&b, h->ev[k + 1], h->ev[k + 2]);
    up += a;
    rb += b;
    k += 2;
  }
  cudaEventElapsedTime(&post, h->ev[k], h->ev[h->n_ev - 1]);
  cudaEventElapsedTime(&tot, h->ev[0], h->ev[h->n_ev - 1]);
  h->stage_ms[0] = pre; h->stage_ms[1] = up; h->stage_ms[2] = rb; h->stage_ms[3] = post; h->stage_ms[4] = tot;
  return GSV_OK;
}

int check_device(int device) {
  int n = 0;
  CUDA_TRY(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return set_err(GSV_E_INVALID_ARG, "device %d out of range (%d devices)", device, n);
  cudaDeviceProp p;
  CUDA_TRY(cudaGetDeviceProperties(&p, device));
  if (p.major != 10)
    return set_err(GSV_E_UNSUPPORTED, "device %d is sm_%d%d; libgsvdec is built for sm_100a (B200)", device, p.major, p.minor);
  return GSV_OK;
}

void destroy_impl(gsvdec* h);
// Frees everything a partly built handle holds when creation fails.
struct HandleDeleter {
  void operator()(gsvdec* h) const { destroy_impl(h); }
};

int create_impl(const gsvdec_tensor* ts, int n, int mode, int device, gsvdec_t** out) {
  if (!out) return set_err(GSV_E_INVALID_ARG, "out is NULL");
  *out = nullptr;
  if (!ts || n <= 0) return set_err(GSV_E_INVALID_ARG, "no tensors given");
  if (mode != GSV_MODE_FP32 && mode != GSV_MODE_BF16 && mode != GSV_MODE_FP32_TC)
    return set_err(GSV_E_INVALID_ARG, "bad mode %d", mode);
  // Validate every tensor first (cheap), then convert and fold all weights in
  // parallel, then pack (the packing jobs also run in parallel, in finish()).
  HostModel m;
  GSV_TRY(load_model(ts, n, m));
  HostFlow hf;
  GSV_TRY(load_flow(ts, n, "flow.flows", hf));
  HostEncp he;
  GSV_TRY(load_encp(ts, n, he));
  {
    std::vector<HostConv*> all{&m.pre, &m.post};
    if (m.has_cond) all.push_back(&m.cond);
    for (auto& u : m.ups) all.push_back(&u);
    for (auto& rb : m.rbs) {
      for (auto& c : rb.c1) all.push_back(&c);
      for (auto& c : rb.c2) all.push_back(&c);
    }
    for (auto& c : hf.layers) {
      for (HostConv* x : {&c.pre, &c.post, &c.cond}) all.push_back(x);
      for (auto& x : c.in) all.push_back(&x);
      for (auto& x : c.rs) all.push_back(&x);
    }
    for (auto& st : he.stacks)
      for (auto& L : st) {
        all.push_back(&L.c1);
        all.push_back(&L.c2);
      }
    if (he.has_proj) all.push_back(&he.proj);
    materialize_all(all);
  }
  GSV_TRY(check_device(device));
  CUDA_TRY(cudaSetDevice(device));
  std::unique_ptr<gsvdec, HandleDeleter> h(new gsvdec());
  h->mode = mode;
  h->device = device;
  h->dt = mode == GSV_MODE_BF16 ? Dt::BF16 : Dt::F32;
  h->x3 = mode == GSV_MODE_FP32_TC;
  h->in_ch = m.pre.d1;
  h->C0 = m.pre.d0;
  h->has_cond = m.has_cond;
  h->gin = m.has_cond ? m.cond.d1 : 0;
  Packer pk{h->dt};
  h->pre = pk.conv(m.pre);
  auto reg = [&](const std::string& n, const GemmConv& g) {
    h->layers[n] = g;
    h->layer_names += n + "\n";
  };
  reg(m.pre.name, h->pre);
  h->hop = 1;
  for (size_t i = 0; i < m.ups.size(); ++i) {
    Stage s;
    s.up = pk.convT(m.ups[i]);
    reg(m.ups[i].name, s.up);
    h->hop *= m.ups[i].stride;
    for (size_t r = 3 * i; r < std::min(3 * i + 3, m.rbs.size()); ++r) {
      std::vector<GemmConv> a, b;
      for (auto& c : m.rbs[r].c1) {
        a.push_back(pk.conv(c));
        reg(c.name, a.back());
      }
      for (auto& c : m.rbs[r].c2) {
        b.push_back(pk.conv(c));
        reg(c.name, b.back());
      }
      s.c1.push_back(std::move(a));
      s.c2.push_back(std::move(b));
    }
    // Summed bias of the branches' last convs (the fused 3-branch op).
    if (s.c2.size() > 1) {
      const int C = s.up.Cout;
      std::vector<float> sum(C, 0.0f);
      for (auto& br : s.c2)
        for (int c = 0; c < C; ++c) sum[c] += pk.biases[br.back().b_off + c];
      // Appended right after the last branch's last bias (see forward_device).
      const size_t expect = s.c2.back().back().b_off + C;
      if (pk.biases.size() != expect) return set_err(GSV_E_SHAPE, "internal bias layout error");
      pk.biases.insert(pk.biases.end(), sum.begin(), sum.end());
    }
    if (h->dt == Dt::BF16 && !s.c2.empty() && !h->ident_off.count(s.up.Cout))
      h->ident_off[s.up.Cout] = pk.identity(s.up.Cout);
    h->stages.push_back(std::move(s));
  }
  if (h->dt == Dt::BF16) {
    // Check every op geometry against the tcgen05 kernel at create time.
    auto ok = [&](const GemmConv& g) {
      TapConv op{};
      op.nseg = 1; op.seg[0].Cin = g.Cin; op.seg[0].ntaps = g.ntaps; op.seg[0].offstep = g.offstep;
      op.seg[0].off0 = g.off0; op.N = g.N; op.Cout = g.Cout;
      return tapconv_tc_supported(op);
    };
    bool all = ok(h->pre);
    for (auto& s : h->stages) {
      all = all && ok(s.up);
      for (auto& br : s.c1) for (auto& g : br) all = all && ok(g);
      for (auto& br : s.c2) for (auto& g : br) all = all && ok(g);
    }
    if (!all) return set_err(GSV_E_UNSUPPORTED, "a layer geometry is not supported by the bf16 tcgen05 kernel");
  }
  // GSV_MODE_FP32_TC: the decoder's convs again, as three-piece K lists in a
  // second arena; biases stay those of the FP32 packing (same offsets).
  Packer px{Dt::BF16};
  px.x3 = true;
  if (h->x3) {
    h->xpre = px.conv(m.pre);
    h->xpre.b_off = h->pre.b_off;
    for (size_t i = 0; i < m.ups.size(); ++i) {
      const Stage& f = h->stages[i];
      Stage s;
      s.up = px.convT(m.ups[i]);
      s.up.b_off = f.up.b_off;
      for (size_t r = 3 * i, br = 0; r < std::min(3 * i + 3, m.rbs.size()); ++r, ++br) {
        std::vector<GemmConv> a, b;
        for (size_t k = 0; k < m.rbs[r].c1.size(); ++k) {
          a.push_back(px.conv(m.rbs[r].c1[k]));
          a.back().b_off = f.c1[br][k].b_off;
        }
        for (size_t k = 0; k < m.rbs[r].c2.size(); ++k) {
          b.push_back(px.conv(m.rbs[r].c2[k]));
          b.back().b_off = f.c2[br][k].b_off;
        }
        s.c1.push_back(std::move(a));
        s.c2.push_back(std::move(b));
      }
      if (!s.c2.empty() && !h->xident_off.count(s.up.Cout)) h->xident_off[s.up.Cout] = px.identity(s.up.Cout);
      h->xstages.push_back(std::move(s));
    }
    auto ok = [&](const GemmConv& g) {
      TapConv op{};
      op.nseg = 2; op.seg[0].Cin = 5 * g.Cin; op.seg[0].pc = g.Cin; op.seg[0].ntaps = g.ntaps;
      op.seg[0].offstep = g.offstep; op.seg[0].off0 = g.off0; op.N = g.N; op.Cout = g.Cout; op.split = 1;
      op.seg[1] = op.seg[0];
      op.seg[1].Cin = g.Cin;
      return tapconv_tc_supported(op);
    };
    bool all = ok(h->xpre);
    for (auto& s : h->xstages) {
      all = all && ok(s.up);
      for (auto& br : s.c1) for (auto& g : br) all = all && ok(g);
      for (auto& br : s.c2) for (auto& g : br) all = all && ok(g);
    }
    if (!all) return set_err(GSV_E_UNSUPPORTED, "a layer geometry is not supported by the three-piece tcgen05 path");
  }
  // The flow (optional), packed into the same weight arena.
  std::vector<std::vector<float>> flow_cond_w, flow_cond_b;
  if (!hf.layers.empty()) {
    GSV_TRY(pack_flow(h.get(), pk, hf, flow_cond_w, flow_cond_b));
    if (h->dt == Dt::BF16) {
      auto ok = [&](const GemmConv& g) {
        TapConv op{};
        op.nseg = 1; op.seg[0].Cin = g.Cin; op.seg[0].ntaps = g.ntaps; op.seg[0].offstep = g.offstep;
        op.seg[0].off0 = g.off0; op.N = g.N; op.Cout = g.Cout;
        return tapconv_tc_supported(op);
      };
      bool all = true;
      for (auto& F : h->flow) {
        all = all && ok(F.pre);
        for (auto& g : F.in) all = all && ok(g);
        for (auto& g : F.res) all = all && ok(g);
        for (auto& g : F.post) all = all && ok(g);
      }
      if (!all) return set_err(GSV_E_UNSUPPORTED, "a flow layer geometry is not supported by the bf16 tcgen05 kernel");
    }
  }
  // The EncP chains (optional), packed into the same weight arena.
  std::vector<float> encp_norm;
  for (int s = 0; s < 3; ++s)
    for (const HostEncpLayer& L : he.stacks[s]) {
      gsvdec::EncpLayer E;
      E.ffn1 = pk.conv(L.c1);
      E.ffn2 = pk.conv(L.c2);
      E.norm = encp_norm.size();
      for (const std::vector<float>* v : {&L.g1, &L.b1, &L.g2, &L.b2}) encp_norm.insert(encp_norm.end(), v->begin(), v->end());
      h->encp_C = L.c1.d1;
      h->encp_F = std::max(h->encp_F, L.c1.d0);
      h->encp[s].push_back(E);
    }
  if (he.has_proj) {
    h->encp_proj = pk.conv(he.proj);
    h->has_encp_proj = true;
    if (!h->encp_C) h->encp_C = he.proj.d1;
  }
  if (h->dt == Dt::BF16 && !encp_norm.empty()) {
    if (!h->ident_off.count(h->encp_C)) h->ident_off[h->encp_C] = pk.identity(h->encp_C);
    auto ok = [&](const GemmConv& g) {
      TapConv op{};
      op.nseg = 1; op.seg[0].Cin = g.Cin; op.seg[0].ntaps = g.ntaps; op.seg[0].offstep = g.offstep;
      op.seg[0].off0 = g.off0; op.N = g.N; op.Cout = g.Cout;
      return tapconv_tc_supported(op);
    };
    bool all = !h->has_encp_proj || ok(h->encp_proj);
    for (int s = 0; s < 3; ++s)
      for (auto& E : h->encp[s]) all = all && ok(E.ffn1) && ok(E.ffn2);
    if (!all) return set_err(GSV_E_UNSUPPORTED, "an enc_p layer geometry is not supported by the bf16 tcgen05 kernel");
  }
  h->layer_names += m.post.name + "\n";
  h->post_K = m.post.K;
  h->post_pad = m.post.pad;
  h->post_C = m.post.d1;
  h->post_bias = m.post.b.empty() ? 0.0f : m.post.b[0];
  if (h->post_C != 16 || h->post_K > 64)
    return set_err(GSV_E_UNSUPPORTED, "conv_post with %d input channels / kernel %d is not supported", h->post_C, h->post_K);
  std::vector<float> post_w((size_t)h->post_K * h->post_C);  // [K][C]
  for (int c = 0; c < h->post_C; ++c)
    for (int j = 0; j < h->post_K; ++j) post_w[(size_t)j * h->post_C + c] = m.post.w[(size_t)c * h->post_K + j];
  // Fill the arena, then upload.
  pk.finish();
  h->w_bytes = pk.size;
  CUDA_TRY(dev_malloc(&h->d_w, std::max<size_t>(h->w_bytes, 256)));
  CUDA_TRY(cudaMemcpy(h->d_w, pk.arena.get(), h->w_bytes, cudaMemcpyHostToDevice));
  if (h->x3) {
    px.finish();
    h->wx_bytes = px.size;
    CUDA_TRY(dev_malloc(&h->d_wx, std::max<size_t>(h->wx_bytes, 256)));
    CUDA_TRY(cudaMemcpy(h->d_wx, px.arena.get(), h->wx_bytes, cudaMemcpyHostToDevice));
  }
  CUDA_TRY(dev_malloc(&h->d_bias, sizeof(float) * std::max<size_t>(pk.biases.size(), 1)));
  CUDA_TRY(cudaMemcpy(h->d_bias, pk.biases.data(), sizeof(float) * pk.biases.size(), cudaMemcpyHostToDevice));
  if (post_w.size() <= sizeof(h->post_wh.w) / sizeof(float)) {
    std::copy(post_w.begin(), post_w.end(), h->post_wh.w);
    h->post_wh_ok = true;
  }
  CUDA_TRY(dev_malloc(&h->d_post_w, sizeof(float) * post_w.size()));
  CUDA_TRY(cudaMemcpy(h->d_post_w, post_w.data(), sizeof(float) * post_w.size(), cudaMemcpyHostToDevice));
  if (h->has_cond) {
    CUDA_TRY(dev_malloc(&h->d_cond_w, sizeof(float) * m.cond.w.size()));
    CUDA_TRY(cudaMemcpy(h->d_cond_w, m.cond.w.data(), sizeof(float) * m.cond.w.size(), cudaMemcpyHostToDevice));
    std::vector<float> cb(h->C0, 0.0f);
    if (!m.cond.b.empty()) cb = m.cond.b;
    CUDA_TRY(dev_malloc(&h->d_cond_b, sizeof(float) * cb.size()));
    CUDA_TRY(cudaMemcpy(h->d_cond_b, cb.data(), sizeof(float) * cb.size(), cudaMemcpyHostToDevice));
  }
  if (!h->flow.empty() && h->flow[0].has_cond) {
    std::vector<float> cw, cb;
    for (size_t l = 0; l < h->flow.size(); ++l) {
      cw.insert(cw.end(), flow_cond_w[l].begin(), flow_cond_w[l].end());
      cb.insert(cb.end(), flow_cond_b[l].begin(), flow_cond_b[l].end());
    }
    CUDA_TRY(dev_malloc(&h->d_flow_cond_w, sizeof(float) * cw.size()));
    CUDA_TRY(cudaMemcpy(h->d_flow_cond_w, cw.data(), sizeof(float) * cw.size(), cudaMemcpyHostToDevice));
    CUDA_TRY(dev_malloc(&h->d_flow_cond_b, sizeof(float) * cb.size()));
    CUDA_TRY(cudaMemcpy(h->d_flow_cond_b, cb.data(), sizeof(float) * cb.size(), cudaMemcpyHostToDevice));
  }
  if (!h->flow.empty()) {
    CUDA_TRY(dev_malloc(&h->d_flow_perm, sizeof(int) * h->flow_perm_host.size()));
    CUDA_TRY(cudaMemcpy(h->d_flow_perm, h->flow_perm_host.data(), sizeof(int) * h->flow_perm_host.size(),
                        cudaMemcpyHostToDevice));
  }
  if (!encp_norm.empty()) {
    CUDA_TRY(dev_malloc(&h->d_encp_norm, sizeof(float) * encp_norm.size()));
    CUDA_TRY(cudaMemcpy(h->d_encp_norm, encp_norm.data(), sizeof(float) * encp_norm.size(),
                        cudaMemcpyHostToDevice));
  }
  CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&h->h_err), sizeof(int), cudaHostAllocMapped));
  *reinterpret_cast<volatile int*>(h->h_err) = 0;
  CUDA_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(&h->d_err), h->h_err, 0));
  for (auto& e : h->ev) CUDA_TRY(cudaEventCreate(&e));
  *out = h.release();
  return GSV_OK;
}

void destroy_impl(gsvdec* h) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(h->device);
  cudaFree(h->d_w);
  cudaFree(h->d_wx);
  cudaFree(h->d_bias);
  cudaFree(h->d_cond_w);
  cudaFree(h->d_cond_b);
  cudaFree(h->d_post_w);
  if (h->h_err) cudaFreeHost(h->h_err);
  cudaFree(h->ws);
  cudaFree(h->lws);
  cudaFree(h->fws);
  cudaFree(h->d_flow_perm);
  cudaFree(h->d_flow_cond_w);
  cudaFree(h->d_flow_cond_b);
  cudaFree(h->d_encp_norm);
  cudaFree(h->ews);
  for (auto& e : h->ev)
    if (e) cudaEventDestroy(e);
  for (auto& run : h->runs)
    for (auto& e : run) cudaEventDestroy(e);
  for (auto& e : h->pool) cudaEventDestroy(e);
  if (h->mstream) cudaStreamDestroy(h->mstream);
  if (h->mev_in) cudaEventDestroy(h->mev_in);
  if (h->mev_done) cudaEventDestroy(h->mev_done);
  for (auto& sl : h->aslot)
    for (cudaEvent_t e : {sl.in_done, sl.comp_done, sl.out_done})
      if (e) cudaEventDestroy(e);
  for (cudaStream_t x : {h->cs_in, h->cs_comp, h->cs_out})
    if (x) cudaStreamDestroy(x);
  if (h->ev_join) cudaEventDestroy(h->ev_join);
  cudaFree(h->aws);
  cudaSetDevice(prev);
  delete h;
}

// A call that uses the decoder workspace from `st` after overlapped calls
// (whose decodes run on cs_comp) is ordered after them.
int join_async(gsvdec* h, cudaStream_t st) {
  if (!h->async_run) return GSV_OK;
  CUDA_TRY(cudaEventRecord(h->ev_join, h->cs_comp));
  CUDA_TRY(cudaStreamWaitEvent(st, h->ev_join, 0));
  h->async_run = false;
  return GSV_OK;
}

// GSV_MEM_HOST_ASYNC: host z / g / lengths / wav, everything queued and the
// call returns.  Call i uses staging slot i % 2:
//   cs_in   waits until the slot's previous call is done with the slot (its
//           output copy ended), then copies z / g / lengths in;
//   cs_comp waits for those copies and until the slot's previous output copy
//           has read its waveform staging, then decodes (the decoder
//           workspace is only ever used from cs_comp, so decodes stay in
//           order);
//   cs_out  waits for the decode and copies the requested samples out;
//   `st`    waits for that copy: the waveform is complete in `st` order.
// The copies of call i thus run while calls i - 1 / i + 1 decode.
int forward_host_async(gsvdec* h, const float* z, const float* g, const int32_t* lengths, int B, int Tsrc,
                       int t_off, int T0, float* wav, cudaStream_t st, int64_t wav_skip, int64_t wav_count) {
  for (cudaStream_t* x : {&h->cs_in, &h->cs_comp, &h->cs_out})
    if (!*x) CUDA_TRY(cudaStreamCreateWithFlags(x, cudaStreamNonBlocking));
  if (!h->ev_join) CUDA_TRY(cudaEventCreateWithFlags(&h->ev_join, cudaEventDisableTiming));
  for (auto& sl : h->aslot)
    for (cudaEvent_t* e : {&sl.in_done, &sl.comp_done, &sl.out_done})
      if (!*e) CUDA_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  const int L = out_len(h, T0);
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t nz = (size_t)B * h->in_ch * T0, ng = (size_t)B * std::max(h->gin, 1), nw = (size_t)B * L;
  const size_t slot = al(nz * 4) + al(ng * 4) + al((size_t)B * 4) + al(nw * 4);
  // Buffers are replaced only once nothing in flight uses them.
  if (2 * slot > h->aws_bytes) {
    for (cudaStream_t x : {h->cs_in, h->cs_comp, h->cs_out}) CUDA_TRY(cudaStreamSynchronize(x));
    if (h->aws) CUDA_TRY(cudaFree(h->aws));
    h->aws = nullptr;
    h->aws_bytes = 0;
    CUDA_TRY(dev_malloc(&h->aws, 2 * slot));
    h->aws_bytes = 2 * slot;
  }
  // Slots keep a fixed stride (half the arena) whatever this call's sizes, so
  // a call never writes into the other slot, whose call may be in flight.
  const size_t stride = h->aws_bytes / 2 / 256 * 256;
  for (int k = 0; k < 2; ++k) {
    char* p = static_cast<char*>(h->aws) + k * stride;
    gsvdec::AsyncSlot& sl = h->aslot[k];
    sl.z = reinterpret_cast<float*>(p);
    sl.g = reinterpret_cast<float*>(p + al(nz * 4));
    sl.len = reinterpret_cast<int*>(p + al(nz * 4) + al(ng * 4));
    sl.wav = reinterpret_cast<float*>(p + al(nz * 4) + al(ng * 4) + al((size_t)B * 4));
  }
  // The decoder workspace (replaced only after the decodes in flight end).
  Workspace w;
  GSV_TRY(ensure_ws(h, B, T0, false, w, h->cs_comp));
  // Join the caller's stream when the workspace was last used from it.
  if (!h->async_run || h->async_stream != st) {
    CUDA_TRY(cudaEventRecord(h->ev_join, st));
    CUDA_TRY(cudaStreamWaitEvent(h->cs_comp, h->ev_join, 0));
    h->async_run = true;
    h->async_stream = st;
  }
  gsvdec::AsyncSlot& sl = h->aslot[h->aseq++ % 2];
  // inputs: the slot is free once its previous call's output copy is done
  // (which follows that call's decode)
  CUDA_TRY(cudaStreamWaitEvent(h->cs_in, sl.out_done, 0));
  if (Tsrc == T0 && t_off == 0)
    CUDA_TRY(cudaMemcpyAsync(sl.z, z, nz * 4, cudaMemcpyHostToDevice, h->cs_in));
  else
    CUDA_TRY(cudaMemcpy2DAsync(sl.z, sizeof(float) * T0, z + t_off, sizeof(float) * Tsrc, sizeof(float) * T0,
                               (size_t)B * h->in_ch, cudaMemcpyHostToDevice, h->cs_in));
  const float* gd = nullptr;
  if (h->has_cond && g) {
    CUDA_TRY(cudaMemcpyAsync(sl.g, g, sizeof(float) * (size_t)B * h->gin, cudaMemcpyHostToDevice, h->cs_in));
    gd = sl.g;
  }
  const int* ld = nullptr;
  if (lengths) {
    CUDA_TRY(cudaMemcpyAsync(sl.len, lengths, sizeof(int) * (size_t)B, cudaMemcpyHostToDevice, h->cs_in));
    ld = sl.len;
  }
  CUDA_TRY(cudaEventRecord(sl.in_done, h->cs_in));
  // decode
  CUDA_TRY(cudaStreamWaitEvent(h->cs_comp, sl.in_done, 0));
  CUDA_TRY(cudaStreamWaitEvent(h->cs_comp, sl.out_done, 0));
  GSV_TRY(forward_device(h, sl.z, T0, 0, gd, ld, B, T0, sl.wav, w, nullptr, h->cs_comp));
  CUDA_TRY(cudaEventRecord(sl.comp_done, h->cs_comp));
  // outputs
  CUDA_TRY(cudaStreamWaitEvent(h->cs_out, sl.comp_done, 0));
  CUDA_TRY(cudaMemcpyAsync(wav, sl.wav + wav_skip, sizeof(float) * (size_t)wav_count, cudaMemcpyDeviceToHost,
                           h->cs_out));
  CUDA_TRY(cudaEventRecord(sl.out_done, h->cs_out));
  CUDA_TRY(cudaStreamWaitEvent(st, sl.out_done, 0));
  return collect_timing(h, h->cs_comp);
}

int forward_impl(gsvdec* h, const float* z, const float* g, const int32_t* lengths, int B,
                 int Tsrc, int t_off, int T0, float* wav, int mem_kind, cudaStream_t st,
                 float* const* taps, int64_t wav_skip, int64_t wav_count) {
  if (!h) return set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (!z || !wav) return set_err(GSV_E_INVALID_ARG, "z and wav must not be NULL");
  if (B <= 0 || T0 <= 0) return set_err(GSV_E_INVALID_ARG, "B=%d and T0=%d must be positive", B, T0);
  if (mem_kind != GSV_MEM_HOST && mem_kind != GSV_MEM_DEVICE && !(mem_kind == GSV_MEM_HOST_ASYNC && !taps))
    return set_err(GSV_E_INVALID_ARG, "bad mem_kind %d", mem_kind);
  if ((int64_t)B * max_act_elems(h, T0) > (int64_t)1 << 40)
    return set_err(GSV_E_INVALID_ARG, "request too large");
  GSV_TRY(take_async_error(h));
  CUDA_TRY(cudaSetDevice(h->device));
  if (mem_kind == GSV_MEM_HOST_ASYNC)
    return forward_host_async(h, z, g, lengths, B, Tsrc, t_off, T0, wav, st, wav_skip, wav_count);
  GSV_TRY(join_async(h, st));
  Workspace w;
  GSV_TRY(ensure_ws(h, B, T0, taps != nullptr, w));
  const int L = out_len(h, T0);
  const float* zd = z;
  const float* gd = (h->has_cond && g) ? g : nullptr;
  const int* ld = lengths;
  float* wd = wav;
  if (mem_kind == GSV_MEM_HOST) {
    // Copy only the requested frames of each channel row: one flat copy when
    // that is all of them, else a pitched copy.
    if (Tsrc == T0 && t_off == 0)
      CUDA_TRY(cudaMemcpyAsync(w.zstage, z, sizeof(float) * (size_t)B * h->in_ch * T0, cudaMemcpyHostToDevice, st));
    else
      CUDA_TRY(cudaMemcpy2DAsync(w.zstage, sizeof(float) * T0, z + t_off, sizeof(float) * Tsrc,
                                 sizeof(float) * T0, (size_t)B * h->in_ch, cudaMemcpyHostToDevice, st));
    zd = w.zstage;
    Tsrc = T0;
    t_off = 0;
    if (gd) {
      CUDA_TRY(cudaMemcpyAsync(w.gstage, g, sizeof(float) * (size_t)B * h->gin, cudaMemcpyHostToDevice, st));
      gd = w.gstage;
    }
    if (lengths) {
      CUDA_TRY(cudaMemcpyAsync(w.lstage, lengths, sizeof(int) * (size_t)B, cudaMemcpyHostToDevice, st));
      ld = w.lstage;
    }
  }
  const bool direct = mem_kind == GSV_MEM_DEVICE && wav_skip == 0 && wav_count == (int64_t)B * L;
  GSV_TRY(forward_device(h, zd, Tsrc, t_off, gd, ld, B, T0, direct ? wd : w.wav, w, taps, st));
  if (!direct) {
    CUDA_TRY(cudaMemcpyAsync(wav, w.wav + wav_skip, sizeof(float) * (size_t)wav_count,
                             mem_kind == GSV_MEM_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, st));
  }
  if (mem_kind == GSV_MEM_HOST || taps) {
    CUDA_TRY(cudaStreamSynchronize(st));
    GSV_TRY(check_device_error(h));
  }
  GSV_TRY(collect_timing(h, st));
  return GSV_OK;
}

// One reference conv layer on [B][Cin][L] fp32 (reference layout) -> [B][Cout][Lout]
// fp32, through the same kernel and packed weights the forward uses: bias
// added, no activation (conv_post: before tanh).
int layer_impl(gsvdec* h, const char* name, const float* x, int B, int L, float* y, int mem_kind,
               cudaStream_t st) {
  if (!name || !x || !y) return set_err(GSV_E_INVALID_ARG, "NULL argument");
  if (B <= 0 || L <= 0) return set_err(GSV_E_INVALID_ARG, "B=%d and L=%d must be positive", B, L);
  if (mem_kind != GSV_MEM_HOST && mem_kind != GSV_MEM_DEVICE)
    return set_err(GSV_E_INVALID_ARG, "bad mem_kind %d", mem_kind);
  const bool post = h->layer_names.find(std::string(name) + "\n") != std::string::npos &&
                    !h->layers.count(name);
  auto it = h->layers.find(name);
  if (!post && it == h->layers.end()) return set_err(GSV_E_INVALID_ARG, "no layer named %s", name);
  const int Cin = post ? h->post_C : it->second.Cin;
  const int Cout = post ? 1 : it->second.Cout;
  const int Lout = post ? L : it->second.Lout(L);
  if (Lout <= 0) return set_err(GSV_E_INVALID_ARG, "output length %d <= 0", Lout);
  GSV_TRY(take_async_error(h));
  CUDA_TRY(cudaSetDevice(h->device));
  const size_t eb = act_bytes(h);
  auto al = [](size_t v) { return (v + 255) / 256 * 256; };
  const size_t nx = (size_t)B * Cin * L, ny = (size_t)B * Cout * Lout;
  const size_t need = al(nx * 4) + al(nx * eb) + al(ny * eb) + al(ny * 4);
  if (need > h->lws_bytes) {
    if (h->lws) CUDA_TRY(cudaFree(h->lws));
    h->lws = nullptr;
    h->lws_bytes = 0;
    CUDA_TRY(dev_malloc(&h->lws, need));
    h->lws_bytes = need;
  }
  char* p = static_cast<char*>(h->lws);
  float* xs = reinterpret_cast<float*>(p);
  void* xt = p + al(nx * 4);
  void* yt = p + al(nx * 4) + al(nx * eb);
  float* ys = reinterpret_cast<float*>(p + al(nx * 4) + al(nx * eb) + al(ny * eb));
  const float* xd = x;
  if (mem_kind == GSV_MEM_HOST) {
    CUDA_TRY(cudaMemcpyAsync(xs, x, nx * 4, cudaMemcpyHostToDevice, st));
    xd = xs;
  }
  h->launches = 0;
  h->n_ev = 0;
  if (h->timing >= 2) {
    cudaEvent_t e;
    if (!h->pool.empty()) {
      e = h->pool.back();
      h->pool.pop_back();
    } else {
      CUDA_TRY(cudaEventCreate(&e));
    }
    CUDA_TRY(cudaEventRecord(e, st));
    h->runs.push_back({e});
    h->run_recs.push_back({});
  }
  CUDA_TRY(launch_transpose_in(xd, B, Cin, L, 0, L, nullptr, xt, h->dt, st));
  GSV_TRY(after_launch(h, st, "input_relayout", 1, 0, 0.0, (4.0 + eb) * nx));
  float* yd = mem_kind == GSV_MEM_DEVICE ? y : ys;
  if (post) {
    CUDA_TRY(launch_post(xt, h->dt, B, L, Cin, h->d_post_w, h->post_wh_ok ? &h->post_wh : nullptr, h->post_K,
                         h->post_pad, h->post_bias,
                         nullptr, xs /* tanh output, unused */, yd, st));
    GSV_TRY(after_launch(h, st, name, 2, 1, 2.0 * Cin * h->post_K * (double)L * B,
                         eb * B * (double)Cin * L + 4.0 * B * (double)L + 4.0 * Cin * h->post_K));
  } else {
    TapConv op = make_op(h, it->second, B, xt, L);
    op.out_raw = yt;
    Work wk;
    wk.add(it->second, B, L, 0, eb);
    GSV_TRY(run_one(h, op, st, name, wk));
    CUDA_TRY(launch_to_ncl(yt, h->dt, B, Lout, Cout, yd, st));
    GSV_TRY(after_launch(h, st, "output_relayout", 1, 0, 0.0, (4.0 + eb) * ny));
  }
  if (mem_kind == GSV_MEM_HOST) {
    CUDA_TRY(cudaMemcpyAsync(y, yd, ny * 4, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    GSV_TRY(check_device_error(h));
  }
  return GSV_OK;
}

// Flow inverse (and, with `decode`, the decoder after it) through host or
// device buffers.
int flow_impl(gsvdec* h, const float* zp, const float* g, const int32_t* lengths, int B, int T0,
              float* out, int mem_kind, cudaStream_t st, bool decode) {
  if (!h) return set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (h->flow.empty()) return set_err(GSV_E_UNSUPPORTED, "this handle was created without flow.flows.* tensors");
  if (!zp || !out) return set_err(GSV_E_INVALID_ARG, "z_p and the output must not be NULL");
  if (B <= 0 || T0 <= 0) return set_err(GSV_E_INVALID_ARG, "B=%d and T0=%d must be positive", B, T0);
  if (mem_kind != GSV_MEM_HOST && mem_kind != GSV_MEM_DEVICE)
    return set_err(GSV_E_INVALID_ARG, "bad mem_kind %d", mem_kind);
  if (decode && h->flow_C != h->in_ch)
    return set_err(GSV_E_SHAPE, "flow width %d != decoder input width %d", h->flow_C, h->in_ch);
  if ((int64_t)B * T0 * std::max(h->flow_C, 2 * h->flow_hid) > (int64_t)1 << 36)
    return set_err(GSV_E_INVALID_ARG, "request too large");
  GSV_TRY(take_async_error(h));
  CUDA_TRY(cudaSetDevice(h->device));
  FlowWs fw;
  GSV_TRY(ensure_flow_ws(h, B, T0, fw));
  const float* zd = zp;
  const float* gd = g;
  const int* ld = lengths;
  if (mem_kind == GSV_MEM_HOST) {
    CUDA_TRY(cudaMemcpyAsync(fw.zstage, zp, sizeof(float) * (size_t)B * h->flow_C * T0, cudaMemcpyHostToDevice, st));
    zd = fw.zstage;
    if (g && h->flow_gin > 0) {
      CUDA_TRY(cudaMemcpyAsync(fw.gstage, g, sizeof(float) * (size_t)B * h->flow_gin, cudaMemcpyHostToDevice, st));
      gd = fw.gstage;
    }
    if (lengths) {
      CUDA_TRY(cudaMemcpyAsync(fw.lstage, lengths, sizeof(int) * (size_t)B, cudaMemcpyHostToDevice, st));
      ld = fw.lstage;
    }
  }
  if (h->flow_gin == 0) gd = nullptr;
  float* zout = (!decode && mem_kind == GSV_MEM_DEVICE) ? out : fw.zout;
  GSV_TRY(flow_device(h, zd, gd, ld, B, T0, zout, fw, st));
  if (!decode) {
    if (mem_kind == GSV_MEM_HOST) {
      CUDA_TRY(cudaMemcpyAsync(out, zout, sizeof(float) * (size_t)B * h->flow_C * T0, cudaMemcpyDeviceToHost, st));
      CUDA_TRY(cudaStreamSynchronize(st));
      GSV_TRY(check_device_error(h));
    }
    return GSV_OK;
  }
  // The decoder reads the same g (src/models/sovits.rs:391-400; gin must match).
  const float* gdec = (h->has_cond && gd && h->gin == h->flow_gin) ? gd : nullptr;
  if (h->has_cond && gd && h->gin != h->flow_gin)
    return set_err(GSV_E_SHAPE, "flow cond width %d != decoder cond width %d", h->flow_gin, h->gin);
  GSV_TRY(join_async(h, st));
  Workspace w;
  GSV_TRY(ensure_ws(h, B, T0, false, w));
  const int L = out_len(h, T0);
  float* wd = mem_kind == GSV_MEM_DEVICE ? out : w.wav;
  GSV_TRY(forward_device(h, zout, T0, 0, gdec, ld, B, T0, wd, w, nullptr, st));
  if (mem_kind == GSV_MEM_HOST) {
    CUDA_TRY(cudaMemcpyAsync(out, wd, sizeof(float) * (size_t)B * L, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    GSV_TRY(check_device_error(h));
  }
  GSV_TRY(collect_timing(h, st));
  return GSV_OK;
}

// ---------------------------------------------------------------------------
// EncP fused elementwise chains.

constexpr float kLayerNormEps = 1e-5f;  // LayerNorm::new (src/utils/weights.rs:419-425)

// Scratch of the EncP entry points: `n` regions of the given byte sizes.
int encp_scratch(gsvdec* h, std::initializer_list<size_t> sizes, std::vector<char*>& out) {
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  size_t need = 0;
  for (size_t b : sizes) need += al(b);
  if (need > h->ews_bytes) {
    if (h->ews) CUDA_TRY(cudaFree(h->ews));
    h->ews = nullptr;
    h->ews_bytes = 0;
    CUDA_TRY(dev_malloc(&h->ews, need));
    h->ews_bytes = need;
  }
  char* p = static_cast<char*>(h->ews);
  out.clear();
  for (size_t b : sizes) {
    out.push_back(p);
    p += al(b);
  }
  return GSV_OK;
}

int encp_common(gsvdec* h, int B, int T, int mem_kind) {
  if (!h) return set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (B <= 0 || T <= 0) return set_err(GSV_E_INVALID_ARG, "B=%d and T=%d must be positive", B, T);
  if (mem_kind != GSV_MEM_HOST && mem_kind != GSV_MEM_DEVICE)
    return set_err(GSV_E_INVALID_ARG, "bad mem_kind %d", mem_kind);
  return take_async_error(h);
}

int encp_layer(gsvdec* h, int stack, int layer, const gsvdec::EncpLayer** L) {
  if (stack < 0 || stack > 2) return set_err(GSV_E_INVALID_ARG, "bad enc_p stack %d", stack);
  if (layer < 0 || layer >= (int)h->encp[stack].size())
    return set_err(GSV_E_INVALID_ARG, "%s has no layer %d (%d loaded)", kEncpStacks[stack], layer,
                   (int)h->encp[stack].size());
  *L = &h->encp[stack][layer];
  return GSV_OK;
}

// Copies `n` values host -> device scratch in host mode; returns the device pointer.
template <typename T>
const T* stage_in(const T* src, size_t n, char* scratch, int mem_kind, cudaStream_t st, int* rc) {
  if (!src || mem_kind == GSV_MEM_DEVICE) return src;
  const cudaError_t e = cudaMemcpyAsync(scratch, src, sizeof(T) * n, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) *rc = set_err(GSV_E_CUDA, "host to device copy failed: %s", cudaGetErrorString(e));
  return reinterpret_cast<const T*>(scratch);
}

int finish_host(gsvdec* h, cudaStream_t st, std::initializer_list<std::pair<float*, const float*>> outs,
                size_t n, int mem_kind) {
  if (mem_kind != GSV_MEM_HOST) return GSV_OK;
  for (const auto& o : outs)
    if (o.first) CUDA_TRY(cudaMemcpyAsync(o.first, o.second, sizeof(float) * n, cudaMemcpyDeviceToHost, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  return check_device_error(h);
}

int encp_add_norm_impl(gsvdec* h, int stack, int layer, int norm, const float* x, const float* y,
                       const int32_t* lengths, int B, int T, float* out, int mem_kind, cudaStream_t st) {
  GSV_TRY(encp_common(h, B, T, mem_kind));
  if (!x || !out) return set_err(GSV_E_INVALID_ARG, "x and out must not be NULL");
  if (norm != 1 && norm != 2) return set_err(GSV_E_INVALID_ARG, "norm must be 1 or 2, got %d", norm);
  const gsvdec::EncpLayer* L = nullptr;
  GSV_TRY(encp_layer(h, stack, layer, &L));
  const int C = h->encp_C;
  const size_t n = (size_t)B * C * T;
  CUDA_TRY(cudaSetDevice(h->device));
  std::vector<char*> sc;
  GSV_TRY(encp_scratch(h, {n * 4, n * 4, n * 4, (size_t)B * 4}, sc));
  int rc = GSV_OK;
  const float* xd = stage_in(x, n, sc[0], mem_kind, st, &rc);
  const float* yd = stage_in(y, n, sc[1], mem_kind, st, &rc);
  const int* ld = stage_in(lengths, (size_t)B, sc[3], mem_kind, st, &rc);
  GSV_TRY(rc);
  float* od = mem_kind == GSV_MEM_DEVICE ? out : reinterpret_cast<float*>(sc[2]);
  begin_run(h, st);
  const float* g = h->d_encp_norm + L->norm + (size_t)(norm - 1) * 2 * C;
  CUDA_TRY(launch_add_layernorm_ncl(xd, yd, g, g + C, B, C, T, kLayerNormEps, ld, od, st));
  GSV_TRY(after_launch(h, st, "encp.add_norm", 1, 0, 0.0, 4.0 * n * (y ? 3 : 2)));
  return finish_host(h, st, {{out, od}}, n, mem_kind);
}

// conv_1 + ReLU, conv_2 + residual, norm2 + x_mask + relayout: the FFN half of
// EncoderLayer::forward on the time-major operand xt ([B][T][C], mode dtype).
int ffn_tail(gsvdec* h, int stack, int layer, const gsvdec::EncpLayer* L, void* xt, void* ht, void* vt,
             const int* lens, int B, int T, float* out, cudaStream_t st) {
  const int C = h->encp_C;
  const double e = (double)act_bytes(h);
  const std::string nm = std::string(kEncpStacks[stack]) + "." + std::to_string(layer);
  {
    // conv_1 + bias + ReLU (LeakyReLU slope 0) in the epilogue.
    TapConv op = make_op(h, L->ffn1, B, xt, T);
    op.out_act = ht;
    op.slope = 0.0f;
    Work wk;
    wk.add(L->ffn1, B, T, 0, e);
    GSV_TRY(run_one(h, op, st, nm + ".conv_1+relu", wk));
  }
  {
    // conv_2 + bias + the residual x.
    TapConv op = make_op(h, L->ffn2, B, ht, T);
    op.res[0] = xt;
    op.nres = 1;
    op.out_raw = vt;
    Work wk;
    wk.add(L->ffn2, B, T, 1, e);
    GSV_TRY(run_one(h, op, st, nm + ".conv_2+res", wk));
  }
  const float* g = h->d_encp_norm + L->norm + 2 * (size_t)C;
  CUDA_TRY(launch_layernorm_tm_ncl(vt, h->dt, B, T, C, g, g + C, kLayerNormEps, lens, out, st));
  return after_launch(h, st, nm + ".norm2+mask", 1, 0, 0.0, (e + 4.0) * (double)B * C * T);
}

// The FFN half alone (x given) or, with `attn`, the whole post-attention
// EncoderLayer::forward: norm1(x + attn) written straight into the GEMM
// operand, then the FFN half.
int encp_ffn_impl(gsvdec* h, int stack, int layer, const float* x, const float* attn, bool with_norm1,
                  const int32_t* lengths, int B, int T, float* out, int mem_kind, cudaStream_t st) {
  GSV_TRY(encp_common(h, B, T, mem_kind));
  if (!x || !out) return set_err(GSV_E_INVALID_ARG, "x and out must not be NULL");
  const gsvdec::EncpLayer* L = nullptr;
  GSV_TRY(encp_layer(h, stack, layer, &L));
  const int C = h->encp_C, F = L->ffn1.Cout;
  if ((int64_t)B * T * F > (int64_t)1 << 34) return set_err(GSV_E_INVALID_ARG, "request too large");
  const size_t n = (size_t)B * C * T, eb = act_bytes(h);
  CUDA_TRY(cudaSetDevice(h->device));
  std::vector<char*> sc;
  GSV_TRY(encp_scratch(h, {n * 4, n * 4, n * eb, (size_t)B * T * F * eb, n * eb, (size_t)B * 4,
                           attn ? n * 4 : 0}, sc));
  int rc = GSV_OK;
  const float* xd = stage_in(x, n, sc[0], mem_kind, st, &rc);
  const float* ad = stage_in(attn, n, sc[6], mem_kind, st, &rc);
  const int* ld = stage_in(lengths, (size_t)B, sc[5], mem_kind, st, &rc);
  GSV_TRY(rc);
  float* od = mem_kind == GSV_MEM_DEVICE ? out : reinterpret_cast<float*>(sc[1]);
  begin_run(h, st);
  const double e = (double)eb;
  if (with_norm1) {
    const float* g = h->d_encp_norm + L->norm;
    CUDA_TRY(launch_add_layernorm_ncl_tm(xd, ad, g, g + C, B, C, T, kLayerNormEps, nullptr, sc[2], h->dt, st));
    GSV_TRY(after_launch(h, st, std::string(kEncpStacks[stack]) + "." + std::to_string(layer) + ".norm1",
                         1, 0, 0.0, (4.0 * (ad ? 2 : 1) + e) * n));
  } else {
    CUDA_TRY(launch_transpose_in(xd, B, C, T, 0, T, nullptr, sc[2], h->dt, st));
    GSV_TRY(after_launch(h, st, "encp.input_relayout", 1, 0, 0.0, (4.0 + e) * n));
  }
  GSV_TRY(ffn_tail(h, stack, layer, L, sc[2], sc[3], sc[4], ld, B, T, od, st));
  return finish_host(h, st, {{out, od}}, n, mem_kind);
}

int encp_speed_len(int T, float speed, int* T_out) {
  if (!T_out) return set_err(GSV_E_INVALID_ARG, "T_out is NULL");
  if (T <= 0) return set_err(GSV_E_INVALID_ARG, "T=%d must be positive", T);
  if (std::fabs(speed - 1.0f) <= FLT_EPSILON) {
    *T_out = T;
    return GSV_OK;
  }
  if (!std::isfinite(speed) || speed <= 0.0f)
    return set_err(GSV_E_INVALID_ARG, "speed must be finite and positive, got %g", (double)speed);
  const float q = (float)T / speed;  // f32 division, then a truncating cast
  if (!(q < 2147483000.0f)) return set_err(GSV_E_INVALID_ARG, "speed %g gives too many frames", (double)speed);
  *T_out = std::max(1, (int)q + 1);
  return GSV_OK;
}

int encp_interp_impl(gsvdec* h, const float* y, int B, int C, int T, int T_out, float* out, int mem_kind,
                     cudaStream_t st) {
  GSV_TRY(encp_common(h, B, T, mem_kind));
  if (!y || !out) return set_err(GSV_E_INVALID_ARG, "y and out must not be NULL");
  if (C <= 0 || T_out <= 0) return set_err(GSV_E_INVALID_ARG, "interpolation length must be positive");
  const size_t ni = (size_t)B * C * T, no = (size_t)B * C * T_out;
  CUDA_TRY(cudaSetDevice(h->device));
  if (T_out == T) {  // the reference returns its input unchanged
    const cudaMemcpyKind k = mem_kind == GSV_MEM_HOST ? cudaMemcpyHostToHost : cudaMemcpyDeviceToDevice;
    CUDA_TRY(cudaMemcpyAsync(out, y, ni * 4, k, st));
    if (mem_kind == GSV_MEM_HOST) CUDA_TRY(cudaStreamSynchronize(st));
    return GSV_OK;
  }
  std::vector<char*> sc;
  GSV_TRY(encp_scratch(h, {ni * 4, no * 4}, sc));
  int rc = GSV_OK;
  const float* yd = stage_in(y, ni, sc[0], mem_kind, st, &rc);
  GSV_TRY(rc);
  float* od = mem_kind == GSV_MEM_DEVICE ? out : reinterpret_cast<float*>(sc[1]);
  begin_run(h, st);
  CUDA_TRY(launch_interpolate(yd, (long long)B * C, T, T_out, od, st));
  GSV_TRY(after_launch(h, st, "encp.interpolate", 1, 0, 0.0, 4.0 * (double)(ni + no)));
  return finish_host(h, st, {{out, od}}, no, mem_kind);
}

int encp_project_impl(gsvdec* h, const float* y, const int32_t* lengths, int B, int T, const float* noise,
                      float noise_scale, float* m, float* logs, float* zp, int mem_kind, cudaStream_t st) {
  GSV_TRY(encp_common(h, B, T, mem_kind));
  if (!h->has_encp_proj) return set_err(GSV_E_UNSUPPORTED, "this handle was created without enc_p.proj");
  if (!y) return set_err(GSV_E_INVALID_ARG, "y must not be NULL");
  if (zp && !noise) return set_err(GSV_E_INVALID_ARG, "z_p needs noise");
  const int C = h->encp_proj.Cin, Co = h->encp_proj.Cout / 2;
  const size_t n = (size_t)B * C * T, no = (size_t)B * Co * T, eb = act_bytes(h);
  CUDA_TRY(cudaSetDevice(h->device));
  std::vector<char*> sc;
  GSV_TRY(encp_scratch(h, {n * 4, n * eb, 2 * no * eb, no * 4, no * 4, no * 4, no * 4, (size_t)B * 4}, sc));
  int rc = GSV_OK;
  const float* yd = stage_in(y, n, sc[0], mem_kind, st, &rc);
  const float* nd = stage_in(noise, no, sc[3], mem_kind, st, &rc);
  const int* ld = stage_in(lengths, (size_t)B, sc[7], mem_kind, st, &rc);
  GSV_TRY(rc);
  const bool dev = mem_kind == GSV_MEM_DEVICE;
  float* md = m ? (dev ? m : reinterpret_cast<float*>(sc[4])) : nullptr;
  float* lsd = logs ? (dev ? logs : reinterpret_cast<float*>(sc[5])) : nullptr;
  float* zd = zp ? (dev ? zp : reinterpret_cast<float*>(sc[6])) : nullptr;
  begin_run(h, st);
  const double e = (double)eb;
  CUDA_TRY(launch_transpose_in(yd, B, C, T, 0, T, nullptr, sc[1], h->dt, st));
  GSV_TRY(after_launch(h, st, "encp.input_relayout", 1, 0, 0.0, (4.0 + e) * n));
  {
    TapConv op = make_op(h, h->encp_proj, B, sc[1], T);
    op.out_raw = sc[2];
    Work wk;
    wk.add(h->encp_proj, B, T, 0, e);
    GSV_TRY(run_one(h, op, st, "enc_p.proj", wk));
  }
  CUDA_TRY(launch_prior_sample(sc[2], h->dt, B, T, Co, ld, nd, noise_scale, md, lsd, zd, st));
  GSV_TRY(after_launch(h, st, "encp.prior_sample", 1, 0, 0.0,
                       2.0 * e * no + 4.0 * no * ((m ? 1 : 0) + (logs ? 1 : 0) + (zp ? 2 : 0))));
  return finish_host(h, st, {{m, md}, {logs, lsd}, {zp, zd}}, no, mem_kind);
}

}  // namespace
}  // namespace gsv

// ---------------------------------------------------------------------------
// C ABI

extern "C" {

const char* gsvdec_last_error(void) { return gsv::g_last_error.c_str(); }

int gsvdec_create(const gsvdec_tensor* tensors, int n_tensors, int mode, int device, gsvdec_t** out) {
  try {
    return gsv::create_impl(tensors, n_tensors, mode, device, out);
  } catch (const std::bad_alloc&) {
    return gsv::set_err(GSV_E_OOM, "host allocation failed");
  } catch (const std::exception& e) {
    return gsv::set_err(GSV_E_INVALID_ARG, "%s", e.what());
  }
}

int gsvdec_create_from_file(const char* path, int mode, int device, gsvdec_t** out) {
  if (!path || !out) return gsv::set_err(GSV_E_INVALID_ARG, "NULL argument");
  try {
    gsv::StFile f;
    std::string err;
    if (!f.open(path, err)) return gsv::set_err(GSV_E_INVALID_ARG, "%s", err.c_str());
    // The decoder's tensors, the flow's and those of the EncP chains (FFN
    // convs, LayerNorms, proj); float dtypes as in src/utils/weights.rs:140-151.
    auto wanted = [](const std::string& k) {
      if (k.compare(0, 4, "dec.") == 0 || k.compare(0, 11, "flow.flows.") == 0) return true;
      if (k.compare(0, 6, "enc_p.") != 0) return false;
      return k.find(".ffn_layers.") != std::string::npos || k.find(".norm_layers_") != std::string::npos ||
             k.compare(0, 11, "enc_p.proj.") == 0;
    };
    std::vector<gsvdec_tensor> ts;
    for (const gsv::StEntry& e : f.entries()) {
      if (!wanted(e.name)) continue;
      gsvdec_tensor t{};
      t.name = e.name.c_str();
      if (e.dtype == "F32") t.dtype = GSV_DTYPE_F32;
      else if (e.dtype == "F16") t.dtype = GSV_DTYPE_F16;
      else if (e.dtype == "BF16") t.dtype = GSV_DTYPE_BF16;
      else return gsv::set_err(GSV_E_DTYPE, "Unsupported dtype %s for %s", e.dtype.c_str(), e.name.c_str());
      if (e.shape.empty() || e.shape.size() > 4)
        return gsv::set_err(GSV_E_SHAPE, "%s: rank %zu not supported", e.name.c_str(), e.shape.size());
      t.ndim = (int)e.shape.size();
      for (int d = 0; d < t.ndim; ++d) t.shape[d] = e.shape[d];
      t.data = e.data;
      ts.push_back(t);
    }
    if (ts.empty()) return gsv::set_err(GSV_E_MISSING_KEY, "no dec.* tensors in %s", path);
    return gsv::create_impl(ts.data(), (int)ts.size(), mode, device, out);
  } catch (const std::bad_alloc&) {
    return gsv::set_err(GSV_E_OOM, "host allocation failed");
  }
}

int gsvdec_destroy(gsvdec_t* h) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  gsv::destroy_impl(h);
  return GSV_OK;
}

int gsvdec_get_info(const gsvdec_t* h, gsvdec_info* info) {
  if (!h || !info) return gsv::set_err(GSV_E_INVALID_ARG, "NULL argument");
  info->mode = h->mode;
  info->device = h->device;
  info->in_channels = h->in_ch;
  info->gin_channels = h->gin;
  info->n_upsamples = (int)h->stages.size();
  int nrb = 0;
  for (auto& s : h->stages) nrb += (int)s.c1.size();
  info->n_resblocks = nrb;
  info->hop = h->hop;
  // Receptive field in input frames: conv_pre pad, then each stage's ConvT
  // taps and resblock halo scaled back by the cumulative stride (rounded up).
  double halo = h->pre.pad;
  double rate = 1.0;
  for (auto& s : h->stages) {
    halo += (double)(s.up.ntaps) / 1.0 / rate;
    rate *= s.up.stride;
    int rbh = 0;
    for (size_t r = 0; r < s.c1.size(); ++r) {
      int hh = 0;
      for (size_t j = 0; j < s.c1[r].size(); ++j)
        hh += (s.c1[r][j].ntaps - 1) * s.c1[r][j].offstep / 2 + (s.c2[r][j].ntaps - 1) / 2;
      rbh = std::max(rbh, hh);
    }
    halo += rbh / rate;
  }
  halo += (double)h->post_pad / rate;
  info->receptive_halo = (int)std::ceil(halo);
  info->weight_bytes = (int64_t)(h->w_bytes + h->wx_bytes);
  return GSV_OK;
}

int gsvdec_forward(gsvdec_t* h, const float* z, const float* g, const int32_t* lengths, int B,
                   int T0, float* wav, int mem_kind, void* stream) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  const int64_t L = gsv::out_len(h, T0 > 0 ? T0 : 1);
  return gsv::forward_impl(h, z, g, lengths, B, T0, 0, T0, wav, mem_kind,
                           static_cast<cudaStream_t>(stream), nullptr, 0, (int64_t)B * L);
}

int gsvdec_forward_chunk(gsvdec_t* h, const float* z, const float* g, int T0, int frame_begin,
                         int frame_end, int halo, float* wav, int mem_kind, void* stream) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (T0 <= 0 || frame_begin < 0 || frame_end > T0 || frame_begin >= frame_end || halo < 0)
    return gsv::set_err(GSV_E_INVALID_ARG, "bad chunk [%d, %d) of %d frames (halo %d)", frame_begin, frame_end, T0, halo);
  const int lo = std::max(0, frame_begin - halo), hi = std::min(T0, frame_end + halo);
  const int64_t skip = (int64_t)(frame_begin - lo) * h->hop;
  const int64_t count = (int64_t)(frame_end - frame_begin) * h->hop;
  return gsv::forward_impl(h, z, g, nullptr, 1, T0, lo, hi - lo, wav, mem_kind,
                           static_cast<cudaStream_t>(stream), nullptr, skip, count);
}

int gsvdec_forward_taps(gsvdec_t* h, const float* z, const float* g, int B, int T0, float* wav,
                        float* const* taps, int n_taps) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (!taps || n_taps != 2 + 2 * (int)h->stages.size())
    return gsv::set_err(GSV_E_INVALID_ARG, "n_taps must be %d", 2 + 2 * (int)h->stages.size());
  const int64_t L = gsv::out_len(h, T0 > 0 ? T0 : 1);
  return gsv::forward_impl(h, z, g, nullptr, B, T0, 0, T0, wav, GSV_MEM_HOST, nullptr, taps, 0,
                           (int64_t)B * L);
}

int gsvdec_flow_info(const gsvdec_t* h, int* n_couplings, int* channels) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (n_couplings) *n_couplings = (int)h->flow.size();
  if (channels) *channels = h->flow_C;
  return GSV_OK;
}

int gsvdec_flow_inverse(gsvdec_t* h, const float* z_p, const float* g, const int32_t* lengths, int B,
                        int T0, float* z, int mem_kind, void* stream) {
  return gsv::flow_impl(h, z_p, g, lengths, B, T0, z, mem_kind, static_cast<cudaStream_t>(stream), false);
}

int gsvdec_flow_decode(gsvdec_t* h, const float* z_p, const float* g, const int32_t* lengths, int B,
                       int T0, float* wav, int mem_kind, void* stream) {
  return gsv::flow_impl(h, z_p, g, lengths, B, T0, wav, mem_kind, static_cast<cudaStream_t>(stream), true);
}

int gsvdec_encp_info(const gsvdec_t* h, int n_layers[3], int* channels, int* filter_channels,
                     int* proj_channels) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (n_layers)
    for (int s = 0; s < 3; ++s) n_layers[s] = (int)h->encp[s].size();
  if (channels) *channels = h->encp_C;
  if (filter_channels) *filter_channels = h->encp_F;
  if (proj_channels) *proj_channels = h->has_encp_proj ? h->encp_proj.Cout : 0;
  return GSV_OK;
}

int gsvdec_encp_add_norm(gsvdec_t* h, int stack, int layer, int norm, const float* x, const float* y,
                         const int32_t* lengths, int B, int T, float* out, int mem_kind, void* stream) {
  return gsv::encp_add_norm_impl(h, stack, layer, norm, x, y, lengths, B, T, out, mem_kind,
                                 static_cast<cudaStream_t>(stream));
}

int gsvdec_encp_ffn(gsvdec_t* h, int stack, int layer, const float* x, const int32_t* lengths, int B,
                    int T, float* out, int mem_kind, void* stream) {
  return gsv::encp_ffn_impl(h, stack, layer, x, nullptr, false, lengths, B, T, out, mem_kind,
                            static_cast<cudaStream_t>(stream));
}

int gsvdec_encp_layer(gsvdec_t* h, int stack, int layer, const float* x, const float* attn,
                      const int32_t* lengths, int B, int T, float* out, int mem_kind, void* stream) {
  return gsv::encp_ffn_impl(h, stack, layer, x, attn, true, lengths, B, T, out, mem_kind,
                            static_cast<cudaStream_t>(stream));
}

int gsvdec_encp_speed_len(int T, float speed, int* T_out) { return gsv::encp_speed_len(T, speed, T_out); }

int gsvdec_encp_interpolate(gsvdec_t* h, const float* y, int B, int C, int T, int T_out, float* out,
                            int mem_kind, void* stream) {
  return gsv::encp_interp_impl(h, y, B, C, T, T_out, out, mem_kind, static_cast<cudaStream_t>(stream));
}

int gsvdec_encp_project(gsvdec_t* h, const float* y, const int32_t* lengths, int B, int T,
                        const float* noise, float noise_scale, float* m, float* logs, float* z_p,
                        int mem_kind, void* stream) {
  return gsv::encp_project_impl(h, y, lengths, B, T, noise, noise_scale, m, logs, z_p, mem_kind,
                                static_cast<cudaStream_t>(stream));
}

int gsvdec_layer_forward(gsvdec_t* h, const char* layer, const float* x, int B, int L, float* y,
                         int mem_kind, void* stream) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  return gsv::layer_impl(h, layer, x, B, L, y, mem_kind, static_cast<cudaStream_t>(stream));
}

int gsvdec_layer_names(const gsvdec_t* h, char* buf, size_t cap, size_t* needed) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (needed) *needed = h->layer_names.size() + 1;
  if (buf && cap) {
    const size_t n = std::min(cap - 1, h->layer_names.size());
    memcpy(buf, h->layer_names.data(), n);
    buf[n] = 0;
  }
  return GSV_OK;
}

int gsvdec_set_stage_timing(gsvdec_t* h, int enable) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (enable < 0 || enable > 2) return gsv::set_err(GSV_E_INVALID_ARG, "timing level must be 0, 1 or 2");
  h->timing = enable;
  return GSV_OK;
}

int gsvdec_get_launch_stats(gsvdec_t* h, gsvdec_launch_stat* out, int max, int* n) {
  if (!h || !n || (max > 0 && !out)) return gsv::set_err(GSV_E_INVALID_ARG, "NULL argument");
  // Fold the pending forwards into per-launch averages (only forwards whose
  // launch sequence matches the last one are averaged), then recycle events.
  if (!h->runs.empty()) {
    CUDA_TRY(cudaSetDevice(h->device));
    const auto& ref = h->run_recs.back();
    std::vector<double> ms(ref.size(), 0.0);
    int used = 0;
    for (size_t k = 0; k < h->runs.size(); ++k) {
      const auto& ev = h->runs[k];
      const auto& rc = h->run_recs[k];
      if (rc.size() != ref.size() || ev.size() != rc.size() + 1) continue;
      bool same = true;
      for (size_t i = 0; i < rc.size() && same; ++i) same = rc[i].name == ref[i].name;
      if (!same) continue;
      CUDA_TRY(cudaEventSynchronize(ev.back()));
      for (size_t i = 0; i < rc.size(); ++i) {
        float t = 0.0f;
        CUDA_TRY(cudaEventElapsedTime(&t, ev[i], ev[i + 1]));
        ms[i] += t;
      }
      used++;
    }
    h->stats.clear();
    for (size_t i = 0; i < ref.size(); ++i) {
      gsvdec_launch_stat s{};
      snprintf(s.name, sizeof s.name, "%s", ref[i].name.c_str());
      s.kind = ref[i].kind;
      s.n_convs = ref[i].nconv;
      s.flops = ref[i].flops;
      s.bytes = ref[i].bytes;
      for (int c = 0; c < 6; ++c) {
        s.conv_flops[c] = ref[i].cf[c];
        s.conv_bytes[c] = ref[i].cb[c];
      }
      s.ms = used ? (float)(ms[i] / used) : 0.0f;
      h->stats.push_back(s);
    }
    for (auto& run : h->runs)
      for (auto& e : run) h->pool.push_back(e);
    h->runs.clear();
    h->run_recs.clear();
  }
  *n = (int)h->stats.size();
  for (int i = 0; i < max && i < *n; ++i) out[i] = h->stats[i];
  return GSV_OK;
}

int gsvdec_get_stage_times(gsvdec_t* h, float ms[5]) {
  if (!h || !ms) return gsv::set_err(GSV_E_INVALID_ARG, "NULL argument");
  for (int i = 0; i < 5; ++i) ms[i] = h->stage_ms[i];
  return GSV_OK;
}

int gsvdec_launch_count(gsvdec_t* h, int B, int T0, int* count) {
  if (!h || !count) return gsv::set_err(GSV_E_INVALID_ARG, "NULL argument");
  (void)B;
  (void)T0;
  *count = h->launches;
  return GSV_OK;
}

int gsvdec_sync_status(gsvdec_t* h, void* stream) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  CUDA_TRY(cudaSetDevice(h->device));
  CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  return gsv::check_device_error(h);
}

int gsvdec_selftest_wait(gsvdec_t* h, int64_t limit_ns, void* stream) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (limit_ns < 1000 || limit_ns > 10000000000ll)
    return gsv::set_err(GSV_E_INVALID_ARG, "limit_ns %lld outside [1e3, 1e10]", (long long)limit_ns);
  GSV_TRY(gsv::take_async_error(h));
  CUDA_TRY(cudaSetDevice(h->device));
  CUDA_TRY(gsv::launch_wait_selftest(h->d_err, (unsigned long long)limit_ns, static_cast<cudaStream_t>(stream)));
  return GSV_OK;
}

int gsvdec_set_alloc_fail_after(int n) {
  gsv::g_alloc_budget.store(n < 0 ? -1 : n);
  return GSV_OK;
}

int gsvdec_workspace_bytes(const gsvdec_t* h, int64_t* bytes) {
  if (!h || !bytes) return gsv::set_err(GSV_E_INVALID_ARG, "NULL argument");
  *bytes = (int64_t)(h->ws_bytes + h->lws_bytes + h->fws_bytes + h->ews_bytes);
  return GSV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free forward (gsvdec_forward_noalloc).
//
// Some callers cannot allocate device memory at call time: a real-time audio
// callback or an inference server whose device memory is carved up by its
// own pool allocator, where a cudaMalloc would block, fragment the pool or
// fail.  For them the forward's per-call scratch (the activation buffers
// between layers) comes from one statically sized device array instead of the
// handle's cudaMalloc'd workspace.  The array is a file-scope __device__
// object, so every GPU that loads this library holds it until process exit.

namespace gsv {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per device
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `device`.  In host code the symbol
// name is only a host-side stand-in, so the address is fetched once per
// device with that device current and cached.
int noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= kMaxDevices)
    return set_err(GSV_E_INVALID_ARG, "device %d out of range for the static scratch", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return set_err(GSV_E_CUDA, "cudaGetSymbolAddress(static scratch) failed on device %d: %s",
                     device, cudaGetErrorString(e));
    g_noalloc_addr[device] = p;
  }
  *out = g_noalloc_addr[device];
  return GSV_OK;
}

// Lays the forward's device-mode buffers out inside [base, base + cap).
int carve_noalloc(const gsvdec* h, int B, int T0, char* base, size_t cap, Workspace& w) {
  const size_t act = max_act_elems(h, T0) * (size_t)B;
  const size_t eb = fwd_act_bytes(h);
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  size_t off = 0;
  const size_t o_zin = off; off += al((size_t)B * T0 * h->in_ch * eb);
  const size_t o_buf = off; off += 12 * al(act * eb);
  const size_t o_bbc = off; off += al((size_t)B * h->C0 * 4);
  const size_t o_len = off; off += al((size_t)B * 16 * 4);
  if (off > cap)
    return set_err(GSV_E_INVALID_ARG,
                   "gsvdec_forward_noalloc: B=%d x T0=%d needs %zu bytes of scratch, the static "
                   "scratch holds %zu bytes",
                   B, T0, off, cap);
  w = Workspace{};
  w.zin = base + o_zin;
  for (int i = 0; i < 12; ++i) w.buf[i] = base + o_buf + i * al(act * eb);
  w.bias_bc = reinterpret_cast<float*>(base + o_bbc);
  w.lens = reinterpret_cast<int*>(base + o_len);
  // FP32 mode: what is left of the array is the split-K scratch (the same
  // split as gsvdec_forward's while it fits, so both give the same samples).
  const size_t part_off = al(off);
  const long long part_floats = h->dt == Dt::F32 && part_off < cap
                                    ? std::min<long long>((long long)((cap - part_off) / 4), kSplitScratchFloats)
                                    : 0;
  w.part = part_floats ? reinterpret_cast<float*>(base + part_off) : nullptr;
  w.part_cap = part_floats;
  return GSV_OK;
}

}  // namespace
}  // namespace gsv

extern "C" int gsvdec_forward_noalloc(gsvdec_t* h, const float* z, const float* g,
                                      const int32_t* lengths, int B, int T0, float* wav,
                                      void* stream) {
  if (!h) return gsv::set_err(GSV_E_INVALID_ARG, "handle is NULL");
  if (!z || !wav) return gsv::set_err(GSV_E_INVALID_ARG, "z and wav must not be NULL");
  if (B <= 0 || T0 <= 0) return gsv::set_err(GSV_E_INVALID_ARG, "B=%d and T0=%d must be positive", B, T0);
  // The same size bound as gsvdec_forward, before any byte count is formed:
  // below it the scratch sizes cannot overflow.
  if ((int64_t)B * gsv::max_act_elems(h, T0) > (int64_t)1 << 40)
    return gsv::set_err(GSV_E_INVALID_ARG,
                        "gsvdec_forward_noalloc: B=%d x T0=%d does not fit the static scratch (%zu bytes)", B, T0,
                        gsv::kNoAllocScratchBytes);
  GSV_TRY(gsv::take_async_error(h));
  {
    const cudaError_t e = cudaSetDevice(h->device);
    if (e != cudaSuccess) return gsv::set_err(GSV_E_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
  }
  void* scratch = nullptr;
  GSV_TRY(gsv::noalloc_scratch(h->device, &scratch));
  gsv::Workspace w;
  GSV_TRY(gsv::carve_noalloc(h, B, T0, static_cast<char*>(scratch), gsv::kNoAllocScratchBytes, w));
  const float* gd = (h->has_cond && g) ? g : nullptr;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  GSV_TRY(gsv::forward_device(h, z, T0, 0, gd, lengths, B, T0, wav, w, nullptr, st));
  // Stage timers, when enabled, are read back exactly as gsvdec_forward does.
  return gsv::collect_timing(h, st);
}

extern "C" int64_t gsvdec_noalloc_scratch_bytes(void) { return (int64_t)gsv::kNoAllocScratchBytes; }

// ---------------------------------------------------------------------------
// Several devices in one call (gsvdec_forward_multi).
//
// Utterances are independent and an output frame depends only on a bounded
// window of input frames, so the decode shards with no exchange step.  A
// batch is split by utterance (longest-processing-time balance of the frame
// counts, then up to kMultiMaxBuckets length buckets per device so short
// utterances are not padded to the longest); one long utterance (B = 1) is
// split into contiguous frame ranges, each decoded with kMultiChunkHalo input
// frames recomputed on both sides.  Every handle runs its share on its own
// stream from its own host thread.  The only transfers are each device's
// inputs in and its waveform pieces out, as copy-engine copies between
// devices (NVLink); no kernel reads another device's memory.  The reference
// decodes on one device (src/config/mod.rs:68-80): no counterpart there.

namespace gsv {
namespace {

constexpr int kMultiMaxBuckets = 8;
constexpr int kMultiBucketOverhead = 300;  // per-forward cost in frames (its launch chain)
constexpr int kMultiChunkHalo = 16;
constexpr int kMultiMaxHandles = 64;

// Utterance indices per worker: longest first onto the least-loaded worker,
// ties to the lower worker; each list ascending.
std::vector<std::vector<int>> plan_utterances(const std::vector<int>& len, const std::vector<int>& ids, int n) {
  std::vector<int> order(ids);
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return len[a] != len[b] ? len[a] > len[b] : a < b; });
  std::vector<long long> load(n, 0);
  std::vector<std::vector<int>> out(n);
  for (int i : order) {
    int r = 0;
    for (int k = 1; k < n; ++k)
      if (load[k] < load[r]) r = k;
    out[r].push_back(i);
    load[r] += len[i];
  }
  for (auto& v : out) std::sort(v.begin(), v.end());
  return out;
}

// Length buckets of one worker's utterances: the split of the length-sorted
// order into at most kMultiMaxBuckets contiguous runs that minimises
// sum(run size x its longest length + kMultiBucketOverhead) (dynamic
// programming; equal-count runs beyond 4096 utterances).  Returns lists of
// utterance ids, each ascending, the buckets by length.
std::vector<std::vector<int>> plan_buckets(const std::vector<int>& len, const std::vector<int>& ids) {
  const int n = (int)ids.size();
  std::vector<std::vector<int>> out;
  if (n == 0) return out;
  std::vector<int> order(ids);
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return len[a] != len[b] ? len[a] < len[b] : a < b; });
  const int K = std::max(1, std::min(kMultiMaxBuckets, n));
  std::vector<int> cuts;  // run boundaries in sorted order: 0 = c0 < c1 < ... = n
  if (n > 4096) {
    for (int k = 0; k <= K; ++k) cuts.push_back((int)((long long)n * k / K));
  } else {
    const double INF = 1e300;
    std::vector<std::vector<double>> best(K + 1, std::vector<double>(n + 1, INF));
    std::vector<std::vector<int>> cut(K + 1, std::vector<int>(n + 1, 0));
    best[0][0] = 0.0;
    for (int k = 1; k <= K; ++k)
      for (int j = 1; j <= n; ++j)
        for (int i = k - 1; i < j; ++i) {
          const double c = best[k - 1][i] + (double)(j - i) * len[order[j - 1]] + kMultiBucketOverhead;
          if (c < best[k][j]) {
            best[k][j] = c;
            cut[k][j] = i;
          }
        }
    int kb = 1;
    for (int k = 2; k <= K; ++k)
      if (best[k][n] < best[kb][n]) kb = k;
    cuts.push_back(n);
    for (int k = kb, j = n; k > 0; --k) {
      j = cut[k][j];
      cuts.push_back(j);
    }
    std::reverse(cuts.begin(), cuts.end());
  }
  for (size_t r = 0; r + 1 < cuts.size(); ++r) {
    if (cuts[r + 1] <= cuts[r]) continue;
    std::vector<int> b(order.begin() + cuts[r], order.begin() + cuts[r + 1]);
    std::sort(b.begin(), b.end());
    out.push_back(std::move(b));
  }
  return out;
}

// One forward of a worker: a masked batch of utterances, or one time chunk.
struct MultiJob {
  std::vector<int> idx;   // utterances (batch job)
  int T = 0;              // frames of the batch: its longest utterance
  int lo = 0, hi = 0;     // chunk job: input window [lo, hi) ...
  int b = 0, e = 0;       // ... and the frames [b, e) it keeps
};

struct MultiCall {
  const float* z;
  const float* g;
  const int32_t* len_user;  // the caller's lengths pointer (or null)
  std::vector<int> len;     // host copy (all T0 without lengths)
  int B, T0, in_ch, gin, hop, mem_kind, dev0;
  float* wav;
  cudaEvent_t ev_in;        // device mode: recorded on the caller's stream
  bool chunked;
};

// Pitched copy of `height` rows of `width` bytes between (possibly) different
// devices, by a copy engine.
cudaError_t copy_rows(void* dst, int ddev, size_t dpitch, const void* src, int sdev, size_t spitch, size_t width,
                      size_t height, cudaStream_t s) {
  if (width == 0 || height == 0) return cudaSuccess;
  const bool flat = height == 1 || (dpitch == width && spitch == width);
  if (ddev == sdev)
    return flat ? cudaMemcpyAsync(dst, src, width * height, cudaMemcpyDeviceToDevice, s)
                : cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDeviceToDevice, s);
  if (flat) return cudaMemcpyPeerAsync(dst, ddev, src, sdev, width * height, s);
  cudaMemcpy3DPeerParms p = {};
  p.srcPtr = make_cudaPitchedPtr(const_cast<void*>(src), spitch, width, height);
  p.srcDevice = sdev;
  p.dstPtr = make_cudaPitchedPtr(dst, dpitch, width, height);
  p.dstDevice = ddev;
  p.extent = make_cudaExtent(width, height, 1);
  return cudaMemcpy3DPeerAsync(&p, s);
}

// Runs of consecutive utterance ids in a sorted list: (position, first id, count).
std::vector<std::array<int, 3>> id_runs(const std::vector<int>& idx) {
  std::vector<std::array<int, 3>> r;
  for (int k = 0; k < (int)idx.size();) {
    int m = 1;
    while (k + m < (int)idx.size() && idx[k + m] == idx[k] + m) ++m;
    r.push_back({k, idx[k], m});
    k += m;
  }
  return r;
}

int multi_worker_device(gsvdec* h, const std::vector<MultiJob>& jobs, const MultiCall& c) {
  CUDA_TRY(cudaSetDevice(h->device));
  if (!h->mstream) CUDA_TRY(cudaStreamCreateWithFlags(&h->mstream, cudaStreamNonBlocking));
  if (!h->mev_done) CUDA_TRY(cudaEventCreateWithFlags(&h->mev_done, cudaEventDisableTiming));
  const cudaStream_t s = h->mstream;
  CUDA_TRY(cudaStreamWaitEvent(s, c.ev_in, 0));
  GSV_TRY(join_async(h, s));
  int maxB = 1, maxT = 1;
  for (const MultiJob& j : jobs) {
    maxB = std::max(maxB, c.chunked ? 1 : (int)j.idx.size());
    maxT = std::max(maxT, c.chunked ? j.hi - j.lo : j.T);
  }
  Workspace w;
  GSV_TRY(ensure_ws(h, maxB, maxT, false, w));  // allocate once for every job
  const bool cond = c.g && h->has_cond;
  const size_t C = c.in_ch;
  for (const MultiJob& j : jobs) {
    if (c.chunked) {
      const int win = j.hi - j.lo;
      GSV_TRY(ensure_ws(h, 1, win, false, w));
      const float* zsrc = c.z;
      int Tsrc = c.T0, toff = j.lo;
      if (h->device != c.dev0) {  // the window [C][win] into this device
        CUDA_TRY(copy_rows(w.zstage, h->device, (size_t)win * 4, c.z + j.lo, c.dev0, (size_t)c.T0 * 4,
                           (size_t)win * 4, C, s));
        zsrc = w.zstage;
        Tsrc = win;
        toff = 0;
      }
      const float* gd = cond ? c.g : nullptr;
      if (cond && h->device != c.dev0) {
        CUDA_TRY(copy_rows(w.gstage, h->device, 0, c.g, c.dev0, 0, (size_t)c.gin * 4, 1, s));
        gd = w.gstage;
      }
      GSV_TRY(forward_device(h, zsrc, Tsrc, toff, gd, nullptr, 1, win, w.wav, w, nullptr, s));
      CUDA_TRY(copy_rows(c.wav + (size_t)j.b * c.hop, c.dev0, 0, w.wav + (size_t)(j.b - j.lo) * c.hop, h->device, 0,
                         (size_t)(j.e - j.b) * c.hop * 4, 1, s));
      continue;
    }
    const int nb = (int)j.idx.size(), T = j.T;
    GSV_TRY(ensure_ws(h, nb, T, false, w));
    const auto runs = id_runs(j.idx);
    for (const auto& r : runs)  // z[u][:, :T] of each utterance -> zstage[k]
      CUDA_TRY(copy_rows(w.zstage + (size_t)r[0] * C * T, h->device, (size_t)T * 4, c.z + (size_t)r[1] * C * c.T0,
                         c.dev0, (size_t)c.T0 * 4, (size_t)T * 4, C * r[2], s));
    const float* gd = nullptr;
    if (cond) {
      for (const auto& r : runs)
        CUDA_TRY(copy_rows(w.gstage + (size_t)r[0] * c.gin, h->device, 0, c.g + (size_t)r[1] * c.gin, c.dev0, 0,
                           (size_t)c.gin * r[2] * 4, 1, s));
      gd = w.gstage;
    }
    const int* ld = nullptr;
    if (c.len_user) {
      std::vector<int> lb(nb);
      for (int k = 0; k < nb; ++k) lb[k] = c.len[j.idx[k]];
      // pageable source: staged by the driver before the call returns
      CUDA_TRY(cudaMemcpyAsync(w.lstage, lb.data(), sizeof(int) * nb, cudaMemcpyHostToDevice, s));
      ld = w.lstage;
    }
    GSV_TRY(forward_device(h, w.zstage, T, 0, gd, ld, nb, T, w.wav, w, nullptr, s));
    const size_t row = (size_t)c.hop * T;  // decoded samples per utterance (zero past its length)
    for (const auto& r : runs)
      CUDA_TRY(copy_rows(c.wav + (size_t)r[1] * c.hop * c.T0, c.dev0, (size_t)c.hop * c.T0 * 4,
                         w.wav + (size_t)r[0] * row, h->device, row * 4, row * 4, r[2], s));
  }
  CUDA_TRY(cudaEventRecord(h->mev_done, s));
  return GSV_OK;
}

int multi_worker_host(gsvdec* h, const std::vector<MultiJob>& jobs, const MultiCall& c) {
  CUDA_TRY(cudaSetDevice(h->device));
  if (!h->mstream) CUDA_TRY(cudaStreamCreateWithFlags(&h->mstream, cudaStreamNonBlocking));
  const cudaStream_t s = h->mstream;
  GSV_TRY(join_async(h, s));
  const bool cond = c.g && h->has_cond;
  const size_t C = c.in_ch;
  std::vector<float> zb, gb, ob;
  for (const MultiJob& j : jobs) {
    if (c.chunked) {
      GSV_TRY(forward_impl(h, c.z, cond ? c.g : nullptr, nullptr, 1, c.T0, j.lo, j.hi - j.lo,
                           c.wav + (size_t)j.b * c.hop, GSV_MEM_HOST, s, nullptr, (int64_t)(j.b - j.lo) * c.hop,
                           (int64_t)(j.e - j.b) * c.hop));
      continue;
    }
    const int nb = (int)j.idx.size(), T = j.T;
    zb.resize((size_t)nb * C * T);
    for (int k = 0; k < nb; ++k)
      for (size_t ch = 0; ch < C; ++ch)
        memcpy(&zb[((size_t)k * C + ch) * T], c.z + ((size_t)j.idx[k] * C + ch) * c.T0, sizeof(float) * T);
    if (cond) {
      gb.resize((size_t)nb * c.gin);
      for (int k = 0; k < nb; ++k)
        memcpy(&gb[(size_t)k * c.gin], c.g + (size_t)j.idx[k] * c.gin, sizeof(float) * c.gin);
    }
    std::vector<int32_t> lb(nb);
    for (int k = 0; k < nb; ++k) lb[k] = c.len[j.idx[k]];
    const size_t row = (size_t)c.hop * T;
    ob.resize((size_t)nb * row);
    GSV_TRY(forward_impl(h, zb.data(), cond ? gb.data() : nullptr, c.len_user ? lb.data() : nullptr, nb, T, 0, T,
                         ob.data(), GSV_MEM_HOST, s, nullptr, 0, (int64_t)nb * row));
    for (int k = 0; k < nb; ++k) {
      float* dst = c.wav + (size_t)j.idx[k] * c.hop * c.T0;
      const size_t valid = (size_t)c.hop * lb[k];
      memcpy(dst, &ob[(size_t)k * row], sizeof(float) * valid);
      memset(dst + valid, 0, sizeof(float) * ((size_t)c.hop * c.T0 - valid));
    }
  }
  return GSV_OK;
}

// Restores the calling thread's current device when the call returns.
struct DeviceGuard {
  int prev = -1;
  DeviceGuard() {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int multi_impl(gsvdec* const* hs, int n, const float* z, const float* g, const int32_t* lengths, int B, int T0,
               float* wav, int mem_kind, cudaStream_t st) {
  if (!hs || n < 1 || n > kMultiMaxHandles)
    return set_err(GSV_E_INVALID_ARG, "need 1..%d handles (got %d)", kMultiMaxHandles, n);
  if (!z || !wav) return set_err(GSV_E_INVALID_ARG, "z and wav must not be NULL");
  if (B <= 0 || T0 <= 0) return set_err(GSV_E_INVALID_ARG, "B=%d and T0=%d must be positive", B, T0);
  if (mem_kind != GSV_MEM_HOST && mem_kind != GSV_MEM_DEVICE)
    return set_err(GSV_E_INVALID_ARG, "bad mem_kind %d", mem_kind);
  gsvdec* h0 = hs[0];
  for (int i = 0; i < n; ++i) {
    if (!hs[i]) return set_err(GSV_E_INVALID_ARG, "handle %d is NULL", i);
    for (int k = 0; k < i; ++k)
      if (hs[k] == hs[i]) return set_err(GSV_E_INVALID_ARG, "handle %d is passed twice", i);
    const gsvdec* h = hs[i];
    if (h->mode != h0->mode || h->in_ch != h0->in_ch || h->gin != h0->gin || h->hop != h0->hop ||
        h->C0 != h0->C0 || h->stages.size() != h0->stages.size() || h->has_cond != h0->has_cond)
      return set_err(GSV_E_INVALID_ARG, "handle %d holds a different model or mode than handle 0", i);
  }
  if ((int64_t)B * max_act_elems(h0, T0) > (int64_t)1 << 40) return set_err(GSV_E_INVALID_ARG, "request too large");
  for (int i = 0; i < n; ++i) GSV_TRY(take_async_error(hs[i]));
  DeviceGuard guard;
  MultiCall c;
  c.z = z;
  c.g = g;
  c.len_user = lengths;
  c.B = B;
  c.T0 = T0;
  c.in_ch = h0->in_ch;
  c.gin = h0->gin;
  c.hop = h0->hop;
  c.mem_kind = mem_kind;
  c.dev0 = h0->device;
  c.wav = wav;
  c.ev_in = nullptr;
  c.len.assign(B, T0);
  CUDA_TRY(cudaSetDevice(c.dev0));
  if (lengths) {
    if (mem_kind == GSV_MEM_HOST) {
      std::copy(lengths, lengths + B, c.len.begin());
    } else {  // the plan needs them on the host: wait for the caller's stream
      CUDA_TRY(cudaMemcpyAsync(c.len.data(), lengths, sizeof(int) * B, cudaMemcpyDeviceToHost, st));
      CUDA_TRY(cudaStreamSynchronize(st));
    }
    for (int b = 0; b < B; ++b)
      if (c.len[b] < 0 || c.len[b] > T0)
        return set_err(GSV_E_INVALID_ARG, "lengths[%d] = %d outside [0, %d]", b, c.len[b], T0);
  }
  // Plan.
  std::vector<std::vector<MultiJob>> jobs(n);
  c.chunked = B == 1 && n > 1 && c.len[0] > 0;
  if (c.chunked) {
    const int L = c.len[0];
    const int base = L / n, extra = L % n;
    for (int r = 0, b = 0; r < n; ++r) {
      const int m = base + (r < extra ? 1 : 0);
      if (m > 0) {
        MultiJob j;
        j.b = b;
        j.e = b + m;
        j.lo = std::max(0, b - kMultiChunkHalo);
        j.hi = std::min(L, b + m + kMultiChunkHalo);
        jobs[r].push_back(j);
      }
      b += m;
    }
  } else {
    std::vector<int> ids;
    for (int b = 0; b < B; ++b)
      if (c.len[b] > 0) ids.push_back(b);
    const auto share = plan_utterances(c.len, ids, n);
    for (int r = 0; r < n; ++r)
      for (auto& bk : plan_buckets(c.len, share[r])) {
        MultiJob j;
        j.T = 0;
        for (int u : bk) j.T = std::max(j.T, c.len[u]);
        j.idx = std::move(bk);
        jobs[r].push_back(std::move(j));
      }
  }
  if (mem_kind == GSV_MEM_DEVICE) {
    if (!h0->mev_in) CUDA_TRY(cudaEventCreateWithFlags(&h0->mev_in, cudaEventDisableTiming));
    CUDA_TRY(cudaEventRecord(h0->mev_in, st));
    c.ev_in = h0->mev_in;
  }
  // Run: one host thread per busy worker (the caller's thread takes the first).
  std::vector<int> rc(n, GSV_OK);
  std::vector<std::string> msg(n);
  auto work = [&](int r) {
    rc[r] = mem_kind == GSV_MEM_DEVICE ? multi_worker_device(hs[r], jobs[r], c) : multi_worker_host(hs[r], jobs[r], c);
    if (rc[r] != GSV_OK) msg[r] = g_last_error;
  };
  std::vector<std::thread> threads;
  int first = -1;
  for (int r = 0; r < n; ++r) {
    if (jobs[r].empty()) continue;
    if (first < 0) first = r;
    else threads.emplace_back(work, r);
  }
  if (first >= 0) work(first);
  for (auto& t : threads) t.join();
  CUDA_TRY(cudaSetDevice(c.dev0));
  for (int r = 0; r < n; ++r)
    if (rc[r] != GSV_OK) return set_err(rc[r], "device %d (handle %d): %s", hs[r]->device, r, msg[r].c_str());
  if (mem_kind == GSV_MEM_DEVICE) {
    for (int r = 0; r < n; ++r)
      if (!jobs[r].empty()) CUDA_TRY(cudaStreamWaitEvent(st, hs[r]->mev_done, 0));
    // Samples past each utterance's length (and all of an empty one) are 0.
    if (lengths) CUDA_TRY(launch_zero_tails(wav, lengths, B, T0, c.hop, st));
  } else {
    for (int b = 0; b < B; ++b) {
      if (c.chunked || c.len[b] == 0) {
        const size_t valid = (size_t)c.hop * c.len[b];
        memset(wav + (size_t)b * c.hop * T0 + valid, 0, sizeof(float) * ((size_t)c.hop * T0 - valid));
      }
    }
  }
  return GSV_OK;
}

}  // namespace
}  // namespace gsv

extern "C" int gsvdec_forward_multi(gsvdec_t* const* handles, int n_handles, const float* z, const float* g,
                                    const int32_t* lengths, int B, int T0, float* wav, int mem_kind,
                                    void* stream) {
  return gsv::multi_impl(handles, n_handles, z, g, lengths, B, T0, wav, mem_kind, static_cast<cudaStream_t>(stream));
}

extern "C" int gsvdec_plan_multi(const int32_t* lengths, int B, int T0, int n_workers, int32_t* worker,
                                 int32_t* bucket) {
  if (!worker || !bucket || B <= 0 || T0 <= 0 || n_workers < 1 || n_workers > gsv::kMultiMaxHandles)
    return gsv::set_err(GSV_E_INVALID_ARG, "bad arguments");
  std::vector<int> len(B, T0);
  if (lengths)
    for (int b = 0; b < B; ++b) {
      if (lengths[b] < 0 || lengths[b] > T0)
        return gsv::set_err(GSV_E_INVALID_ARG, "lengths[%d] = %d outside [0, %d]", b, lengths[b], T0);
      len[b] = lengths[b];
    }
  std::vector<int> ids;
  for (int b = 0; b < B; ++b) {
    worker[b] = -1;
    bucket[b] = -1;
    if (len[b] > 0) ids.push_back(b);
  }
  const auto share = gsv::plan_utterances(len, ids, n_workers);
  for (int r = 0; r < n_workers; ++r) {
    const auto bks = gsv::plan_buckets(len, share[r]);
    for (int k = 0; k < (int)bks.size(); ++k)
      for (int u : bks[k]) {
        worker[u] = r;
        bucket[u] = k;
      }
  }
  return GSV_OK;
}
