// Host executor and C ABI (include/llx.h) of the B200 integer-datapath backend.
//
// Model load parses qgraph.json (DIALECT.md section 2), validates every op the way the
// golden model and the C++ runtime do (golden.py:246-342, host.cpp:47-130) plus the
// operand ranges the kernels rely on, uploads qweights.bin once, and compiles the op list
// into a step plan:
//   * QUANT ops are fused into the RMSNorm / RoPE step that produces their input;
//   * the K half of KV_WRITE is fused into the RoPE(+QUANT) step of the keys;
//   * every other op is one kernel.
// A session owns the KV cache of B independent sequences and an activation arena whose
// buffers are reused by liveness (or kept per name for activation dumps).  The M=1
// decode step is captured once into a CUDA graph; POS lives in device memory so the same
// graph replays at every position, and the argmax of one step feeds the next on the
// device.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "../../include/llx.h"
#include "collective.h"
#include "json.hpp"
#include "kernels.h"
#include "launch.cuh"
#include "luts_data.h"
#include "numerics.cuh"

namespace llx {

static thread_local std::string g_err;

// error text of llx_linear_argmax_noalloc (noalloc.cu), read back by llx_last_error
void noalloc_set_error(const std::string& msg) { g_err = msg; }

struct Error : std::runtime_error {
  llx_status code;
  Error(llx_status c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define LLX_CUDA(x)                                                                                         \
  do {                                                                                                      \
    cudaError_t e_ = (x);                                                                                   \
    if (e_ != cudaSuccess)                                                                                  \
      throw Error(e_ == cudaErrorMemoryAllocation ? LLX_ERR_OOM : LLX_ERR_CUDA,                             \
                  std::string(#x) + ": " + cudaGetErrorString(e_));                                         \
  } while (0)

static void require(bool ok, llx_status code, const std::string& msg) {
  if (!ok) throw Error(code, msg);
}

// ---------------------------------------------------------------------------------------
// qgraph model
// ---------------------------------------------------------------------------------------
enum class DT { I8, I16, I32, RQ };

struct TensorSpec {
  DT dt;
  std::vector<int64_t> shape;
  int64_t offset = 0, count = 0, bytes = 0;
};

struct ActInfo {
  std::string name;
  int cols = 0;
  int elem = 2;
};

enum class SK {
  Embed, RmsNorm, Quant, Linear, Rope, KvWrite, Attention, Add, Mul, Silu, LinearGroup, Gated, RopeGroup,
  // tensor parallelism (graphs from llaccel_b200.tp.shard): int32 partial sums of a row-split
  // linear, their in-place all-reduce, and the requant + epilogue of the reduced sums
  LinearPartial, AllReduce, Requant
};

struct Step {
  SK kind;
  int in = -1, in2 = -1, out = -1, out2 = -1;  // activation ids
  int64_t w_off = -1, rq_off = -1, bias_off = -1, gamma_off = -1;
  int narrow = 0;  // linear: |acc + bias| < 2^31 always
  int N = 0, K = 0, heads = 1, H = 0, Hkv = 0, D = 0, layer = -1;
  int out_i8 = 0, epi = 0, aux_shift = 0, silu_Si = 0, silu_sh = 0;
  int64_t silu_Mi = 0;
  int64_t eps_t = 0, C = 0;
  int sh_post = 0;
  int64_t Mq = 0;
  int Sq = 0;
  bool write_k = false, write_v = true;
  int64_t Ms = 0, Mo = 0;
  int Ss = 0, So = 0, prob_bits = 8;
  int sh = 0;
  std::string label;
  // fused steps: the constituent steps (executed one by one when the fused kernel does not
  // apply, e.g. on the CUDA-core GEMM path) and the concatenated / interleaved weights
  std::vector<Step> parts;
  int nseg = 0;
  // decode (M = 1): a RoPE group folded into the following attention step (attention ->
  // index of that RoPE group step; the RoPE group -> folded)
  int rope_step = -1;
  bool folded = false;
  int seg_start[5] = {0, 0, 0, 0, 0};
};

static std::vector<int> step_outs(const Step& x) {
  std::vector<int> v;
  if (!x.parts.empty()) {
    for (const Step& p : x.parts)
      for (int a : step_outs(p)) v.push_back(a);
    return v;
  }
  for (int a : {x.out, x.out2})
    if (a >= 0) v.push_back(a);
  return v;
}

static std::vector<int> step_ins(const Step& x) {
  std::vector<int> v;
  if (!x.parts.empty()) {
    std::vector<int> made;
    for (const Step& p : x.parts) {
      for (int a : step_ins(p))
        if (std::find(made.begin(), made.end(), a) == made.end() && std::find(v.begin(), v.end(), a) == v.end())
          v.push_back(a);  // each activation once, however many constituents read it
      for (int a : step_outs(p)) made.push_back(a);
    }
    return v;
  }
  for (int a : {x.in, x.in2})
    if (a >= 0) v.push_back(a);
  return v;
}

static bool writes_kv(const Step& x) {
  if (x.kind == SK::Attention || x.kind == SK::KvWrite || x.kind == SK::RopeGroup) return true;
  return x.kind == SK::Rope && x.write_k;
}

struct LayerKV {
  int Hkv = 0, D = 0;
};

}  // namespace llx

struct llx_model {
  int device = 0;
  llx_opts opts{};
  int dim = 0, n_layers = 0, n_heads = 0, n_kv_heads = 0, head_dim = 0, ffn = 0, vocab = 0, vocab_padded = 0;
  int max_seq = 0, prefill_m = 16, E_RES = 0, E_LOGIT = 0;
  int n_ops = 0;
  std::unordered_map<std::string, llx::TensorSpec> tensors;
  std::vector<llx::ActInfo> acts;
  std::unordered_map<std::string, int> act_id;
  std::vector<llx::Step> steps;
  std::map<int, llx::LayerKV> kv_layers;  // qgraph layer id -> geometry
  int input_act = 0, output_act = -1;
  int tail_start = 0;
  std::vector<int> tail_inputs;
  std::vector<int> act_uses;  // steps that read each activation (fused groups count once)
  int64_t embed_off = -1, cos_off = -1, sin_off = -1;
  int embed_rows = 0;
  std::vector<uint8_t> blob_host_check;  // unused after upload
  size_t blob_bytes = 0;
  uint8_t* d_blob = nullptr;
  uint16_t* d_luts = nullptr;  // numerics.cuh kLut* layout
  int sms = 148;
  // tensor parallelism: this rank's vocabulary shard is global channels
  // [vocab_base, vocab_base + vocab_padded) of vocab_padded_full; tp = null on one GPU
  int tp_rank = 0, tp_world = 1, vocab_base = 0, vocab_padded_full = 0;
  llx::TpComm* tp = nullptr;
  int n_sessions = 0;
};

namespace llx {

static std::string read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  require(f.good(), LLX_ERR_IO, "cannot open " + path);
  std::ostringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

static int64_t ival(const json::Value& op, const char* key) {
  const json::Value* v = op.find(key);
  require(v && v->kind == json::Value::Number && v->is_int, LLX_ERR_INVALID,
          std::string("op field '") + key + "' missing or not an integer");
  return v->i;
}
static int64_t ival_or(const json::Value& op, const char* key, int64_t dflt) {
  const json::Value* v = op.find(key);
  if (!v || v->is_null()) return dflt;
  require(v->kind == json::Value::Number && v->is_int, LLX_ERR_INVALID,
          std::string("op field '") + key + "' is not an integer");
  return v->i;
}
static std::string sval(const json::Value& op, const char* key) {
  const json::Value* v = op.find(key);
  require(v && v->kind == json::Value::String, LLX_ERR_INVALID, std::string("op field '") + key + "' missing");
  return v->s;
}
static std::string sval_or(const json::Value& op, const char* key, const std::string& dflt) {
  const json::Value* v = op.find(key);
  if (!v || v->is_null()) return dflt;
  require(v->kind == json::Value::String, LLX_ERR_INVALID, std::string("op field '") + key + "' is not a string");
  return v->s;
}
static void check_shift(int64_t s, const std::string& what) {
  require(s >= 0 && s <= 63, LLX_ERR_INVALID, what + ": shift " + std::to_string(s) + " outside [0, 63]");
}
static void check_mult(int64_t m, const std::string& what) {
  require(m >= 0 && m <= 0xFFFFFFFFll, LLX_ERR_INVALID, what + ": multiplier " + std::to_string(m) + " outside [0, 2^32)");
}

static const TensorSpec& tensor(llx_model* m, const std::string& name, DT dt, const std::string& ctx) {
  auto it = m->tensors.find(name);
  require(it != m->tensors.end(), LLX_ERR_INVALID, ctx + ": unknown tensor '" + name + "'");
  require(it->second.dt == dt, LLX_ERR_INVALID, ctx + ": tensor '" + name + "' has the wrong dtype");
  return it->second;
}

static int act_lookup(llx_model* m, const std::string& name, const std::string& ctx) {
  auto it = m->act_id.find(name);
  require(it != m->act_id.end(), LLX_ERR_INVALID, ctx + ": activation '" + name + "' is not produced before use");
  return it->second;
}

static int act_define(llx_model* m, const std::string& name, int cols, int elem) {
  require(cols > 0, LLX_ERR_INVALID, "activation '" + name + "' has no columns");
  auto it = m->act_id.find(name);
  if (it != m->act_id.end()) {
    // the golden model overwrites a re-defined name; the plan keeps one buffer per name
    ActInfo& a = m->acts[it->second];
    require(a.cols == cols && a.elem == elem, LLX_ERR_UNSUPPORTED,
            "activation '" + name + "' redefined with a different shape");
    return it->second;
  }
  m->acts.push_back(ActInfo{name, cols, elem});
  m->act_id[name] = (int)m->acts.size() - 1;
  return (int)m->acts.size() - 1;
}

static void load_tensors(llx_model* m, const json::Value& g, size_t blob_size) {
  for (auto& kv : g.at("tensors").obj) {
    const json::Value& spec = kv.second;
    TensorSpec t;
    const std::string& d = spec.at("dtype").as_str();
    int elem;
    if (d == "i8") {
      t.dt = DT::I8;
      elem = 1;
    } else if (d == "i16") {
      t.dt = DT::I16;
      elem = 2;
    } else if (d == "i32") {
      t.dt = DT::I32;
      elem = 4;
    } else if (d == "rq") {
      t.dt = DT::RQ;
      elem = 8;
    } else {
      throw Error(LLX_ERR_INVALID, "tensor '" + kv.first + "': unknown dtype " + d);
    }
    int64_t count = 1;
    for (auto& s : spec.at("shape").arr) {
      const int64_t v = s.as_int();
      require(v >= 0, LLX_ERR_INVALID, "tensor '" + kv.first + "': negative extent");
      t.shape.push_back(v);
      count *= v;
    }
    t.count = count;
    t.bytes = count * elem;
    t.offset = spec.at("offset").as_int();
    require(t.offset >= 0 && (size_t)(t.offset + t.bytes) <= blob_size, LLX_ERR_INVALID,
            "tensor '" + kv.first + "' lies outside the weight file");
    require(t.offset % 16 == 0, LLX_ERR_UNSUPPORTED, "tensor '" + kv.first + "' is not 16-byte aligned");
    m->tensors[kv.first] = t;
  }
}

// validates one rq table: M in [0, 2^32), S in [0, 63] for every channel
static void check_rq_table(const std::vector<uint8_t>& blob, const TensorSpec& t, const std::string& ctx) {
  const int32_t* p = reinterpret_cast<const int32_t*>(blob.data() + t.offset);
  for (int64_t n = 0; n < t.count; ++n) {
    require(p[2 * n] >= 0, LLX_ERR_INVALID, ctx + ": negative requant multiplier at channel " + std::to_string(n));
    check_shift(p[2 * n + 1], ctx + " channel " + std::to_string(n));
  }
}

// rq table, bias, out_dtype and epilogue of a linear (or of the requant of a row-split
// linear's reduced sums) over N channels; returns max |bias|
static int64_t parse_rq_epilogue(llx_model* m, const json::Value& op, Step& s, const std::vector<uint8_t>& blob,
                                 const std::string& ctx);

static int64_t append_blob(std::vector<uint8_t>& blob, const void* src, size_t n) {
  const size_t off = (blob.size() + 63) & ~size_t(63);
  blob.resize(off + n);
  std::memcpy(blob.data() + off, src, n);
  return (int64_t)off;
}

// Multi-output GEMM over the row-concatenation of the parts' weights (same input, epilogue
// none).  Segment boundaries stay 16-channel aligned so no epilogue chunk straddles two.
static bool make_linear_group(std::vector<uint8_t>& blob, const std::vector<Step>& parts, Step* out) {
  if (parts.size() < 2 || parts.size() > 4) return false;
  const int K = parts[0].K;
  int N = 0;
  bool any_bias = false;
  for (const Step& p : parts) {
    if (p.kind != SK::Linear || p.epi != EPI_NONE || p.K != K || p.in != parts[0].in || p.N % 16) return false;
    N += p.N;
    any_bias |= p.bias_off >= 0;
  }
  std::vector<int8_t> w((size_t)N * K);
  std::vector<int32_t> rq((size_t)N * 2), bias((size_t)N, 0);
  Step g;
  g.kind = SK::LinearGroup;
  g.in = parts[0].in;
  g.K = K;
  g.N = N;
  g.nseg = (int)parts.size();
  int n0 = 0;
  int64_t max_bias = 0;
  for (size_t i = 0; i < parts.size(); ++i) {
    const Step& p = parts[i];
    g.seg_start[i] = n0;
    std::memcpy(w.data() + (size_t)n0 * K, blob.data() + p.w_off, (size_t)p.N * K);
    std::memcpy(rq.data() + (size_t)n0 * 2, blob.data() + p.rq_off, (size_t)p.N * 8);
    if (p.bias_off >= 0) {
      std::memcpy(bias.data() + n0, blob.data() + p.bias_off, (size_t)p.N * 4);
      for (int j = 0; j < p.N; ++j) max_bias = std::max<int64_t>(max_bias, std::llabs((long long)bias[n0 + j]));
    }
    n0 += p.N;
  }
  g.seg_start[parts.size()] = N;
  g.narrow = (int64_t)K * 16384 + max_bias < (1ll << 31) ? 1 : 0;
  g.w_off = append_blob(blob, w.data(), w.size());
  g.rq_off = append_blob(blob, rq.data(), rq.size() * 4);
  g.bias_off = any_bias ? append_blob(blob, bias.data(), bias.size() * 4) : -1;
  g.parts = parts;
  g.label = "linear_group:" + parts[0].label;
  *out = g;
  return true;
}

// Gate/up pair (+ the quant of their product): weights, requant pairs and biases
// interleaved in 16-row blocks (gate block j, up block j), one GEMM of 2N channels.
static bool make_gated(std::vector<uint8_t>& blob, const std::vector<Step>& parts, Step* out) {
  const Step& gs = parts[0];
  const Step& us = parts[1];
  if (gs.N % 16 || gs.N != us.N || gs.K != us.K) return false;
  const int N = gs.N, K = gs.K;
  std::vector<int8_t> w((size_t)2 * N * K);
  std::vector<int32_t> rq((size_t)4 * N), bias((size_t)2 * N, 0);
  const bool any_bias = gs.bias_off >= 0 || us.bias_off >= 0;
  int64_t max_bias = 0;
  for (int blk = 0; blk < N / 16; ++blk) {
    for (int h = 0; h < 2; ++h) {
      const Step& p = h ? us : gs;
      const size_t dst_row = (size_t)blk * 32 + h * 16, src_row = (size_t)blk * 16;
      std::memcpy(w.data() + dst_row * K, blob.data() + p.w_off + src_row * K, (size_t)16 * K);
      std::memcpy(rq.data() + dst_row * 2, blob.data() + p.rq_off + src_row * 8, 16 * 8);
      if (p.bias_off >= 0) {
        std::memcpy(bias.data() + dst_row, blob.data() + p.bias_off + src_row * 4, 16 * 4);
        for (int j = 0; j < 16; ++j) max_bias = std::max<int64_t>(max_bias, std::llabs((long long)bias[dst_row + j]));
      }
    }
  }
  Step g;
  g.kind = SK::Gated;
  g.in = gs.in;
  g.K = K;
  g.N = 2 * N;
  g.narrow = (int64_t)K * 16384 + max_bias < (1ll << 31) ? 1 : 0;
  g.w_off = append_blob(blob, w.data(), w.size());
  g.rq_off = append_blob(blob, rq.data(), rq.size() * 4);
  g.bias_off = any_bias ? append_blob(blob, bias.data(), bias.size() * 4) : -1;
  g.parts = parts;
  g.label = "gated:" + us.label;
  *out = g;
  return true;
}

// Second plan pass: multi-output q/k/v GEMMs, gate/up pairs, and the per-layer RoPE group.
static void fuse_steps(llx_model* m, std::vector<uint8_t>& blob) {
  std::vector<Step>& st = m->steps;
  std::vector<Step> out;
  size_t i = 0;
  while (i < st.size()) {
    const Step& x = st[i];
    if (x.kind == SK::Linear && x.epi == EPI_NONE) {
      size_t j = i + 1;
      while (j < st.size() && st[j].kind == SK::Linear && st[j].epi == EPI_NONE && st[j].in == x.in && st[j].K == x.K)
        ++j;
      Step grp;
      if (j - i >= 2 && make_linear_group(blob, std::vector<Step>(st.begin() + i, st.begin() + j), &grp)) {
        out.push_back(grp);
        i = j;
        continue;
      }
    }
    if (x.kind == SK::Linear && x.epi == EPI_SILU && !x.out_i8 && i + 1 < st.size()) {
      const Step& u = st[i + 1];
      if (u.kind == SK::Linear && u.epi == EPI_MUL && u.in == x.in && u.in2 == x.out && !u.out_i8) {
        std::vector<Step> parts{x, u};
        if (i + 2 < st.size() && st[i + 2].kind == SK::Quant && st[i + 2].in == u.out) parts.push_back(st[i + 2]);
        Step grp;
        if (make_gated(blob, parts, &grp)) {
          out.push_back(grp);
          i += parts.size();
          continue;
        }
      }
    }
    if (x.kind == SK::Rope && !x.write_k && x.out2 >= 0 && i + 2 < st.size()) {
      const Step& k = st[i + 1];
      const Step& v = st[i + 2];
      if (k.kind == SK::Rope && k.write_k && k.out2 >= 0 && k.D == x.D && v.kind == SK::KvWrite && v.in < 0 &&
          v.layer == k.layer && v.Hkv == k.H && v.D == k.D) {
        Step grp;
        grp.kind = SK::RopeGroup;
        grp.parts = {x, k, v};
        grp.layer = k.layer;
        grp.D = x.D;
        grp.label = "rope_group:" + x.label;
        out.push_back(grp);
        i += 3;
        continue;
      }
    }
    out.push_back(x);
    ++i;
  }
  st.swap(out);
}

static int64_t parse_rq_epilogue(llx_model* m, const json::Value& op, Step& s, const std::vector<uint8_t>& blob,
                                 const std::string& ctx) {
  const TensorSpec& rq = tensor(m, sval(op, "rq"), DT::RQ, ctx);
  require(rq.count == s.N, LLX_ERR_INVALID, ctx + ": rq table size != N");
  check_rq_table(blob, rq, ctx);
  s.rq_off = rq.offset;
  const std::string bias = sval_or(op, "bias", "");
  int64_t max_bias = 0;
  if (!bias.empty()) {
    const TensorSpec& b = tensor(m, bias, DT::I32, ctx);
    require(b.count == s.N, LLX_ERR_INVALID, ctx + ": bias size != N");
    s.bias_off = b.offset;
    const int32_t* bp = reinterpret_cast<const int32_t*>(blob.data() + b.offset);
    for (int64_t n = 0; n < b.count; ++n) max_bias = std::max<int64_t>(max_bias, std::llabs((long long)bp[n]));
  }
  const std::string od = sval_or(op, "out_dtype", "i16");
  const std::string ep = sval_or(op, "epilogue", "none");
  require(od == "i16" || od == "i8", LLX_ERR_INVALID, ctx + ": unknown out_dtype " + od);
  s.out_i8 = od == "i8";
  if (s.out_i8) require(ep == "none", LLX_ERR_INVALID, "i8 output is only valid with epilogue none");
  if (ep == "none") {
    s.epi = EPI_NONE;
  } else if (ep == "resadd" || ep == "mul") {
    s.epi = ep == "resadd" ? EPI_RESADD : EPI_MUL;
    s.in2 = act_lookup(m, sval(op, "aux"), ctx);
    require(m->acts[s.in2].elem == 2 && m->acts[s.in2].cols == s.N, LLX_ERR_INVALID, ctx + ": aux must be i16 [M][N]");
    s.aux_shift = (int)ival_or(op, "aux_shift", 0);
    check_shift(s.aux_shift, ctx);
  } else if (ep == "silu") {
    s.epi = EPI_SILU;
    const json::Value& sp = op.at("silu");
    s.silu_Mi = ival(sp, "Mi");
    s.silu_Si = (int)ival(sp, "Si");
    s.silu_sh = (int)ival(sp, "sh_out");
    check_mult(s.silu_Mi, ctx);
    check_shift(s.silu_Si, ctx);
    check_shift(s.silu_sh, ctx);
  } else {
    throw Error(LLX_ERR_INVALID, "unknown epilogue '" + ep + "'");
  }
  return max_bias;
}

static void build_plan(llx_model* m, const json::Value& g, std::vector<uint8_t>& blob) {
  const json::Value& ops = g.at("ops");
  require(ops.kind == json::Value::Array, LLX_ERR_INVALID, "qgraph 'ops' is not a list");
  m->n_ops = (int)ops.arr.size();
  const std::string in_name = g.find("input") ? g.at("input").as_str() : "input";
  const std::string out_name = g.find("output") ? g.at("output").as_str() : "logits";
  m->input_act = act_define(m, in_name, m->dim, 2);
  const bool fuse = m->opts.fuse != 0;

  // producer op index for each output name, to decide QUANT fusion
  std::unordered_map<std::string, int> producer;
  for (size_t i = 0; i < ops.arr.size(); ++i) {
    const json::Value& op = ops.arr[i];
    const std::string k = sval(op, "op");
    if (k != "kv_write") producer[sval(op, "out")] = (int)i;
  }
  std::vector<int> fused_into(ops.arr.size(), -1);  // quant op -> producer op index
  std::vector<int> quant_of(ops.arr.size(), -1);    // producer op -> fused quant op
  if (fuse) {
    for (size_t i = 0; i < ops.arr.size(); ++i) {
      const json::Value& op = ops.arr[i];
      if (sval(op, "op") != "quant") continue;
      auto it = producer.find(sval(op, "in"));
      if (it == producer.end()) continue;
      const int p = it->second;
      const std::string pk = sval(ops.arr[p], "op");
      if ((pk == "rmsnorm" || pk == "rope") && quant_of[p] < 0 && p < (int)i) {
        fused_into[i] = p;
        quant_of[p] = (int)i;
      }
    }
  }

  Step emb;
  emb.kind = SK::Embed;
  emb.out = m->input_act;
  emb.label = "embed";
  m->steps.push_back(emb);
  std::unordered_map<int, size_t> step_of_op;

  for (size_t i = 0; i < ops.arr.size(); ++i) {
    const json::Value& op = ops.arr[i];
    const std::string k = sval(op, "op");
    const std::string ctx = "op " + std::to_string(i) + " (" + k + ")";
    Step s;
    s.label = k + ":" + (k == "kv_write" ? std::string("layer") + std::to_string(ival(op, "layer")) : sval(op, "out"));
    if (k == "rmsnorm") {
      s.kind = SK::RmsNorm;
      s.in = act_lookup(m, sval(op, "in"), ctx);
      require(m->acts[s.in].elem == 2, LLX_ERR_INVALID, ctx + ": input must be i16");
      const TensorSpec& gm = tensor(m, sval(op, "gamma"), DT::I16, ctx);
      require(gm.shape.size() == 1, LLX_ERR_INVALID, ctx + ": gamma must be 1-D");
      s.K = (int)gm.shape[0];
      s.heads = (int)ival_or(op, "heads", 1);
      require(s.heads >= 1 && m->acts[s.in].cols == s.heads * s.K, LLX_ERR_INVALID, "RMSNorm head geometry mismatch");
      require(ival_or(op, "K", s.K) == s.K, LLX_ERR_INVALID, ctx + ": K does not match gamma");
      require(s.K % 8 == 0 && s.K <= 65536, LLX_ERR_UNSUPPORTED, ctx + ": K must be a multiple of 8 and <= 65536");
      s.gamma_off = gm.offset;
      s.eps_t = ival(op, "eps_t");
      s.C = ival(op, "C");
      require(s.eps_t >= 0 && s.eps_t < (1ll << 32), LLX_ERR_INVALID, ctx + ": eps_t outside u32");
      require(s.C >= 0 && s.C < (1ll << 40), LLX_ERR_INVALID, ctx + ": C out of range");
      s.sh_post = (int)ival(op, "sh_post");
      check_shift(s.sh_post, ctx);
      s.out = act_define(m, sval(op, "out"), m->acts[s.in].cols, 2);
    } else if (k == "quant") {
      const int64_t M = ival(op, "M"), S = ival(op, "S");
      check_mult(M, ctx);
      check_shift(S, ctx);
      const int in = act_lookup(m, sval(op, "in"), ctx);
      require(m->acts[in].elem == 2, LLX_ERR_INVALID, ctx + ": input must be i16");
      const int out = act_define(m, sval(op, "out"), m->acts[in].cols, 1);
      if (fused_into[i] >= 0) {
        Step& p = m->steps[step_of_op.at(fused_into[i])];
        p.out2 = out;
        p.Mq = M;
        p.Sq = (int)S;
        continue;
      }
      s.kind = SK::Quant;
      s.in = in;
      s.out = out;
      s.Mq = M;
      s.Sq = (int)S;
    } else if (k == "linear" || k == "linear_partial") {
      s.kind = k == "linear" ? SK::Linear : SK::LinearPartial;
      s.in = act_lookup(m, sval(op, "in"), ctx);
      require(m->acts[s.in].elem == 1, LLX_ERR_INVALID, ctx + ": linear input must be i8");
      const TensorSpec& w = tensor(m, sval(op, "w"), DT::I8, ctx);
      s.N = (int)ival(op, "N");
      s.K = (int)ival(op, "K");
      require(w.shape.size() == 2 && w.shape[0] == s.N && w.shape[1] == s.K && m->acts[s.in].cols == s.K,
              LLX_ERR_INVALID, k + " " + sval(op, "out") + ": shapes do not match N/K");
      require(s.K % 16 == 0 && s.N % 8 == 0, LLX_ERR_UNSUPPORTED, ctx + ": N must be a multiple of 8, K of 16");
      s.w_off = w.offset;
      if (s.kind == SK::LinearPartial) {
        s.out = act_define(m, sval(op, "out"), s.N, 4);
      } else {
        const int64_t max_bias = parse_rq_epilogue(m, op, s, blob, ctx);
        // |sum_k a*w| <= K * 128 * 128; the bias add stays in 32 bits when the total cannot wrap
        s.narrow = (int64_t)s.K * 16384 + max_bias < (1ll << 31) ? 1 : 0;
        s.out = act_define(m, sval(op, "out"), s.N, s.out_i8 ? 1 : 2);
      }
    } else if (k == "allreduce") {
      s.kind = SK::AllReduce;
      s.in = act_lookup(m, sval(op, "in"), ctx);
      require(m->acts[s.in].elem == 4, LLX_ERR_INVALID, ctx + ": all-reduce input must be int32 partial sums");
      require(sval(op, "out") == sval(op, "in"), LLX_ERR_UNSUPPORTED, ctx + ": the all-reduce is in place (out == in)");
      require(sval_or(op, "reduce", "sum") == "sum", LLX_ERR_UNSUPPORTED, ctx + ": only sum all-reduces exist");
      s.N = m->acts[s.in].cols;
      s.out = s.in;
    } else if (k == "requant") {
      s.kind = SK::Requant;
      s.in = act_lookup(m, sval(op, "in"), ctx);
      s.N = (int)ival(op, "N");
      require(m->acts[s.in].elem == 4 && m->acts[s.in].cols == s.N, LLX_ERR_INVALID,
              ctx + ": requant input must be int32 [M][N]");
      require(s.N % 8 == 0, LLX_ERR_UNSUPPORTED, ctx + ": N must be a multiple of 8");
      parse_rq_epilogue(m, op, s, blob, ctx);
      s.out = act_define(m, sval(op, "out"), s.N, s.out_i8 ? 1 : 2);
    } else if (k == "rope") {
      s.kind = SK::Rope;
      s.in = act_lookup(m, sval(op, "in"), ctx);
      s.H = (int)ival(op, "H");
      s.D = (int)ival(op, "D");
      require(s.H >= 1 && s.D >= 2 && s.D % 2 == 0 && m->acts[s.in].cols == s.H * s.D && m->acts[s.in].elem == 2,
              LLX_ERR_INVALID, ctx + ": RoPE geometry mismatch");
      require(m->cos_off >= 0, LLX_ERR_INVALID, ctx + ": rope tables missing");
      const TensorSpec& ct = m->tensors.at("rope_cos");
      require(ct.shape.size() == 2 && ct.shape[0] >= m->max_seq && ct.shape[1] == s.D / 2, LLX_ERR_INVALID,
              ctx + ": rope table shape does not cover [max_seq][D/2]");
      s.out = act_define(m, sval(op, "out"), s.H * s.D, 2);
    } else if (k == "kv_write") {
      s.kind = SK::KvWrite;
      s.layer = (int)ival(op, "layer");
      s.Hkv = (int)ival(op, "Hkv");
      s.D = (int)ival(op, "D");
      s.in = act_lookup(m, sval(op, "k"), ctx);
      s.in2 = act_lookup(m, sval(op, "v"), ctx);
      require(s.Hkv >= 1 && s.D >= 16 && s.D % 16 == 0, LLX_ERR_UNSUPPORTED, ctx + ": head_dim must be a multiple of 16");
      require(m->acts[s.in].elem == 1 && m->acts[s.in2].elem == 1 && m->acts[s.in].cols == s.Hkv * s.D &&
                  m->acts[s.in2].cols == s.Hkv * s.D,
              LLX_ERR_INVALID, ctx + ": k/v must be i8 [M][Hkv*D]");
      auto it = m->kv_layers.find(s.layer);
      if (it != m->kv_layers.end())
        require(it->second.Hkv == s.Hkv && it->second.D == s.D, LLX_ERR_INVALID, ctx + ": layer geometry changed");
      m->kv_layers[s.layer] = LayerKV{s.Hkv, s.D};
      // K half fused into the producing RoPE step when its QUANT was fused there
      if (fuse) {
        const std::string kname = sval(op, "k");
        auto pit = producer.find(kname);
        if (pit != producer.end() && sval(ops.arr[pit->second], "op") == "quant" && fused_into[pit->second] >= 0) {
          const int rope_op = fused_into[pit->second];
          if (sval(ops.arr[rope_op], "op") == "rope") {
            Step& rs = m->steps[step_of_op.at(rope_op)];
            if (rs.H == s.Hkv && rs.D == s.D) {
              rs.write_k = true;
              rs.layer = s.layer;
              s.in = -1;  // V only
            }
          }
        }
      }
    } else if (k == "attention") {
      s.kind = SK::Attention;
      s.layer = (int)ival(op, "layer");
      s.H = (int)ival(op, "H");
      s.Hkv = (int)ival(op, "Hkv");
      s.D = (int)ival(op, "D");
      s.in = act_lookup(m, sval(op, "q"), ctx);
      require(s.Hkv >= 1 && s.H % s.Hkv == 0, LLX_ERR_INVALID, ctx + ": H must be a multiple of Hkv");
      require(m->acts[s.in].elem == 1 && m->acts[s.in].cols == s.H * s.D, LLX_ERR_INVALID, ctx + ": q must be i8 [M][H*D]");
      auto it = m->kv_layers.find(s.layer);
      require(it != m->kv_layers.end(), LLX_ERR_INVALID, ctx + ": attention before the layer's kv_write");
      require(it->second.Hkv == s.Hkv && it->second.D == s.D, LLX_ERR_INVALID, ctx + ": KV geometry mismatch");
      s.Ms = ival(op, "Ms");
      s.Ss = (int)ival(op, "Ss");
      s.Mo = ival(op, "Mo");
      s.So = (int)ival(op, "So");
      check_mult(s.Ms, ctx);
      check_mult(s.Mo, ctx);
      check_shift(s.Ss, ctx);
      check_shift(s.So, ctx);
      s.prob_bits = (int)ival_or(op, "prob_bits", 8);
      require(s.prob_bits == 8 || s.prob_bits == 15, LLX_ERR_INVALID, "attention prob_bits must be 8 or 15");
      s.out = act_define(m, sval(op, "out"), s.H * s.D, 1);
    } else if (k == "add" || k == "mul") {
      s.kind = k == "add" ? SK::Add : SK::Mul;
      s.in = act_lookup(m, sval(op, "a"), ctx);
      s.in2 = act_lookup(m, sval(op, "b"), ctx);
      require(m->acts[s.in].elem == 2 && m->acts[s.in2].elem == 2 && m->acts[s.in].cols == m->acts[s.in2].cols,
              LLX_ERR_INVALID, ctx + ": operands must be i16 of equal width");
      s.sh = (int)ival(op, k == "add" ? "sh_b" : "sh");
      check_shift(s.sh, ctx);
      s.out = act_define(m, sval(op, "out"), m->acts[s.in].cols, 2);
    } else if (k == "silu") {
      s.kind = SK::Silu;
      s.in = act_lookup(m, sval(op, "in"), ctx);
      require(m->acts[s.in].elem == 2, LLX_ERR_INVALID, ctx + ": input must be i16");
      s.silu_Mi = ival(op, "Mi");
      s.silu_Si = (int)ival(op, "Si");
      s.silu_sh = (int)ival(op, "sh_out");
      check_mult(s.silu_Mi, ctx);
      check_shift(s.silu_Si, ctx);
      check_shift(s.silu_sh, ctx);
      s.out = act_define(m, sval(op, "out"), m->acts[s.in].cols, 2);
    } else {
      throw Error(LLX_ERR_INVALID, "unknown qgraph op '" + k + "'");
    }
    step_of_op[i] = m->steps.size();
    m->steps.push_back(s);
  }
  if (fuse) fuse_steps(m, blob);
  auto it = m->act_id.find(out_name);
  require(it != m->act_id.end(), LLX_ERR_INVALID, "qgraph output '" + out_name + "' is never produced");
  m->output_act = it->second;
  m->act_uses.assign(m->acts.size(), 0);
  for (const Step& x : m->steps)
    for (int a : step_ins(x)) m->act_uses[a]++;
  m->act_uses[m->output_act]++;
  // a RoPE group directly before the attention it feeds folds into the decode attention when
  // nothing else reads its rotated rows (the quantized q goes only to the attention)
  for (size_t i = 1; i < m->steps.size(); ++i) {
    Step& at = m->steps[i];
    Step& rg = m->steps[i - 1];
    if (at.kind != SK::Attention || rg.kind != SK::RopeGroup || rg.parts.size() != 3) continue;
    const Step& q = rg.parts[0];
    const Step& k = rg.parts[1];
    const Step& v = rg.parts[2];
    const bool ok = q.out2 == at.in && m->act_uses[at.in] == 1 && m->act_uses[q.out] == 0 &&
                    m->act_uses[k.out] == 0 && (k.out2 < 0 || m->act_uses[k.out2] == 0) && k.layer == at.layer &&
                    v.layer == at.layer && q.D == at.D && k.H == at.Hkv && q.H == at.H && v.in2 >= 0 &&
                    m->acts[v.in2].elem == 1 && (at.D == 16 || at.D == 32 || at.D == 64 || at.D == 128 || at.D == 256);
    if (ok) {
      at.rope_step = (int)i - 1;
      rg.folded = true;
    }
  }
  require(m->acts[m->output_act].elem == 2 && m->acts[m->output_act].cols == m->vocab_padded, LLX_ERR_INVALID,
          "output must be i16 [M][vocab_padded]");
  // row-independent tail: everything after the last attention / KV write
  int last = 0;
  for (size_t i = 0; i < m->steps.size(); ++i)
    if (writes_kv(m->steps[i])) last = (int)i;
  m->tail_start = last + 1;
  std::vector<char> seen(m->acts.size(), 0);
  for (size_t i = m->tail_start; i < m->steps.size(); ++i) {
    for (int a : step_ins(m->steps[i])) {
      if (seen[a]) continue;
      bool defined_in_tail = false;
      for (size_t j = m->tail_start; j < i; ++j)
        for (int o : step_outs(m->steps[j]))
          if (o == a) defined_in_tail = true;
      if (!defined_in_tail) {
        seen[a] = 1;
        m->tail_inputs.push_back(a);
      }
    }
  }
}

static void load_model(llx_model* m, const std::string& dir) {
  const std::string text = read_file(dir + "/qgraph.json");
  json::Value g;
  try {
    g = json::parse(text);
  } catch (const std::exception& e) {
    throw Error(LLX_ERR_INVALID, std::string("qgraph.json: ") + e.what());
  }
  const json::Value& md = g.at("model");
  m->dim = (int)md.at("dim").as_int();
  m->n_layers = (int)md.at("n_layers").as_int();
  m->n_heads = (int)ival_or(md, "n_heads", 0);
  m->n_kv_heads = (int)ival_or(md, "n_kv_heads", 0);
  m->head_dim = (int)ival_or(md, "head_dim", 0);
  m->ffn = (int)ival_or(md, "ffn", 0);
  m->vocab = (int)md.at("vocab").as_int();
  m->vocab_padded = (int)ival_or(md, "vocab_padded", m->vocab);
  m->max_seq = (int)md.at("max_seq").as_int();
  m->prefill_m = (int)ival_or(md, "prefill_m", 16);
  m->E_RES = (int)md.at("E_RES").as_int();
  m->E_LOGIT = (int)md.at("E_LOGIT").as_int();
  require(m->prefill_m >= 1 && m->prefill_m <= 16 && m->max_seq % m->prefill_m == 0, LLX_ERR_INVALID,
          "max_seq must be divisible by prefill_m in [1,16]");
  require(m->dim > 0 && m->dim % 16 == 0, LLX_ERR_UNSUPPORTED, "dim must be a positive multiple of 16");
  m->vocab_padded_full = m->vocab_padded;
  if (const json::Value* tp = md.find("tp")) {
    // a rank graph of a tensor-parallel group: the output is this rank's vocabulary shard
    m->tp_rank = (int)ival(*tp, "rank");
    m->tp_world = (int)ival(*tp, "world");
    m->vocab_base = (int)ival(*tp, "vocab_offset");
    m->vocab_padded_full = (int)ival(*tp, "vocab_padded_full");
    require(m->tp_world >= 1 && m->tp_rank >= 0 && m->tp_rank < m->tp_world, LLX_ERR_INVALID, "model.tp: bad rank/world");
    require(m->vocab_base >= 0 && m->vocab_base + m->vocab_padded <= m->vocab_padded_full, LLX_ERR_INVALID,
            "model.tp: vocabulary shard outside vocab_padded_full");
  }
  require(m->vocab > 0 && m->vocab <= m->vocab_padded_full, LLX_ERR_INVALID, "vocab exceeds vocab_padded");
  const std::string wfile = g.find("weights_file") ? g.at("weights_file").as_str() : "qweights.bin";
  std::vector<uint8_t> blob;
  {
    const std::string b = read_file(dir + "/" + wfile);
    blob.assign(b.begin(), b.end());
  }
  m->blob_bytes = blob.size();
  load_tensors(m, g, blob.size());
  {
    const TensorSpec& e = tensor(m, "embed", DT::I16, "model");
    require(e.shape.size() == 2 && e.shape[1] == m->dim && e.shape[0] >= m->vocab, LLX_ERR_INVALID,
            "embed must be [>=vocab][dim]");
    m->embed_off = e.offset;
    m->embed_rows = (int)e.shape[0];
    m->cos_off = tensor(m, "rope_cos", DT::I16, "model").offset;
    m->sin_off = tensor(m, "rope_sin", DT::I16, "model").offset;
    require(m->tensors.at("rope_cos").shape == m->tensors.at("rope_sin").shape, LLX_ERR_INVALID,
            "rope tables differ in shape");
  }
  build_plan(m, g, blob);
  LLX_CUDA(cudaSetDevice(m->device));
  LLX_CUDA(cudaMalloc(&m->d_blob, std::max<size_t>(blob.size(), 256)));
  LLX_CUDA(cudaMemcpy(m->d_blob, blob.data(), blob.size(), cudaMemcpyHostToDevice));
  {
    uint16_t tab[kLutCount];
    std::memcpy(tab + kLutSig, kSig, sizeof(kSig));
    std::memcpy(tab + kLutExpI, kExpI, sizeof(kExpI));
    std::memcpy(tab + kLutExpF, kExpF, sizeof(kExpF));
    LLX_CUDA(cudaMalloc(&m->d_luts, sizeof(tab)));
    LLX_CUDA(cudaMemcpy(m->d_luts, tab, sizeof(tab), cudaMemcpyHostToDevice));
  }
  LLX_CUDA(cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, m->device));
  if (m->opts.gemm_path == 0 || m->opts.gemm_path >= 3) {
    int major = 0;
    LLX_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, m->device));
    require(major == 10, LLX_ERR_UNSUPPORTED, "the tensor-core path needs an sm_100 (B200) device");
    LLX_CUDA(prepare_linear_tc());
  }
  size_t att_smem = 0;
  for (const Step& x : m->steps)
    if (x.kind == SK::Attention)
      att_smem = std::max({att_smem, attention_smem_bytes(x.H, x.Hkv, x.D, m->max_seq),
                           attention_decode_smem_bytes(x.H, x.Hkv, x.D, m->max_seq)});
  if (att_smem) {
    int optin = 0;
    LLX_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device));
    require(att_smem <= (size_t)optin, LLX_ERR_UNSUPPORTED,
            "attention needs " + std::to_string(att_smem) + " B of shared memory for max_seq; the device allows " +
                std::to_string(optin));
    LLX_CUDA(prepare_attention(att_smem));
    for (const Step& x : m->steps)
      if (x.kind == SK::Attention) LLX_CUDA(prepare_attention_decode(x.H, x.Hkv, x.D, m->max_seq));
  }
}

}  // namespace llx

// ---------------------------------------------------------------------------------------
// Session
// ---------------------------------------------------------------------------------------
struct llx_session {
  llx_model* m = nullptr;
  int B = 0, max_rows = 0;
  bool keep = false;
  cudaStream_t st = nullptr;
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<size_t> act_off;      // per activation
  std::vector<size_t> tail_off;     // gathered copies of the tail inputs
  int8_t* kv = nullptr;
  size_t kv_bytes = 0;
  std::map<int, std::pair<int8_t*, int8_t*>> kv_layer;  // layer -> (K, V) caches [B][Hkv][max_seq][D]
  int32_t* d_tokens = nullptr;
  int32_t* d_pos = nullptr;
  int32_t* d_step = nullptr;
  int32_t* d_err = nullptr;
  int32_t* d_rec = nullptr;
  int32_t* d_argmax = nullptr;
  int32_t* d_hist = nullptr;
  int hist_cap = 0;
  int max_tail_rows = 0;  // rows per sequence the row-independent tail can hold
  // pinned staging: tokens / record rows / argmax [B*max_rows], pos word, lazily sized i16
  int32_t* h_tok = nullptr;
  int32_t* h_rec = nullptr;
  int32_t* h_am = nullptr;
  int32_t* h_pos = nullptr;
  int16_t* h_i16 = nullptr;
  size_t h_i16_n = 0;
  std::vector<size_t> act_rows;  // allocated rows of each activation buffer
  size_t tail_rows_alloc = 0;
  std::map<std::tuple<const void*, int64_t, int64_t, int>, CUtensorMap> tmaps;
  int32_t* d_fault = nullptr;  // nonzero: a tensor-core pipeline wait timed out
  unsigned long long* d_amax_key = nullptr;  // [B*max_rows] fused argmax keys of the output linear
  int16_t* d_gather = nullptr;  // tensor parallelism: all-gathered logits shards [world][rows][vocab_padded]
  size_t gather_n = 0;
  // decode-step graphs: [0] records only the argmax (the output linear stores no logits),
  // [1] also stores the logits rows
  cudaGraphExec_t decode_exec[2] = {nullptr, nullptr};
  int decode_launches = 0;
  // the output linear stores its logits (cleared while a logits-free decode graph is captured
  // or profiled; the fused argmax keys are produced either way)
  bool store_logits = true;
  int last_R = 0, last_Rtail = 0;
  bool last_tail = false;
  bool last_logits = true;  // the last launch stored its logits rows
  uint8_t* d_flush = nullptr;  // profiling: a buffer twice the L2 size, written between timed launches
};

namespace llx {

static void* dptr(llx_model* m, int64_t off) { return off < 0 ? nullptr : m->d_blob + off; }

struct Binding {
  std::vector<void*> p;
  std::vector<size_t> rows;  // allocated rows behind p[i]
};

static Binding bind(llx_session* s, bool tail_mode) {
  Binding b;
  b.p.resize(s->m->acts.size());
  b.rows.resize(s->m->acts.size());
  for (size_t i = 0; i < s->m->acts.size(); ++i) {
    b.p[i] = s->arena + s->act_off[i];
    b.rows[i] = s->act_rows[i];
  }
  (void)tail_mode;
  return b;
}

static const CUtensorMap& tmap(llx_session* s, const void* base, int64_t rows, int64_t K, int box) {
  auto key = std::make_tuple(base, rows, K, box);
  auto it = s->tmaps.find(key);
  if (it != s->tmaps.end()) return it->second;
  CUtensorMap mp;
  const cudaError_t e = make_tmap_i8(&mp, base, rows, K, box);
  if (e != cudaSuccess) throw Error(LLX_ERR_CUDA, std::string("tensor map encode failed: ") + cudaGetErrorString(e));
  return s->tmaps.emplace(key, mp).first->second;
}

// Tensor-core tiling for R rows x N channels x K: the widest channel tile that alone
// covers the SMs; else the widest tile that does with K split across a cluster (each CTA
// keeping at least two 128-byte K blocks); else the narrowest tile, deepest such split.
static void pick_tc_tiling(int R, int N, int K, int sms, int* nt, int* ksplit) {
  const int row_tiles = (R + 127) / 128;
  const int nkb = (K + 127) / 128;
  const int cands[5] = {256, 128, 64, 32, 16};
  for (int c : cands) {
    if ((N + c - 1) / c * row_tiles >= sms) {
      *nt = c;
      *ksplit = 1;
      return;
    }
  }
  for (int c : cands) {
    const int tiles = (N + c - 1) / c * row_tiles;
    for (int ks = 2; ks <= 8 && nkb / ks >= 2; ks *= 2) {
      if (tiles * ks >= sms) {
        *nt = c;
        *ksplit = ks;
        return;
      }
    }
  }
  *nt = 16;
  int ks = 1;
  while (ks < 8 && nkb / (ks * 2) >= 2) ks *= 2;
  *ksplit = ks;
}

// An RMSNorm (with its fused quant) followed by the linear that reads its quantized row: the
// pair the one-row GEMV runs as one kernel, the norm in its prologue.  Needs the quantized
// row read by that linear alone and the i16 row by nobody.
static bool norm_pair(const llx_model* m, size_t i) {
  if (i + 1 >= m->steps.size()) return false;
  const Step& n = m->steps[i];
  const Step& g = m->steps[i + 1];
  if (n.kind != SK::RmsNorm || n.heads != 1 || n.out2 < 0 || n.K % 16 || n.K > 16384) return false;
  if (!(g.kind == SK::Linear || g.kind == SK::LinearGroup || g.kind == SK::Gated)) return false;
  return g.in == n.out2 && g.K == n.K && m->act_uses[n.out2] == 1 && m->act_uses[n.out] == 0;
}

static int gemm_path_for(const llx_model* m, int R);

// The pair is run as one kernel in this launch: one row (batch-1 decode), the CUDA-core GEMV
// path, activations not kept for dumps.
static bool norm_folds_into_next(const llx_session* s, size_t i, int R) {
  return R == 1 && !s->keep && gemm_path_for(s->m, R) == 1 && norm_pair(s->m, i);
}

static int enqueue_one(llx_session* s, const Binding& bd, const Step& x, int R, int M);

// One tensor-core GEMM over R rows of activation `in` (N x K weights at a.W).  Many output
// tiles (at least two per SM: prefill, the vocabulary projection) go to the persistent
// kernel, whose epilogue overlaps the next tile's main loop; otherwise the per-tile kernel
// with the widest tile that fills the SMs, or split-K clusters when the tiles are too few.
static cudaError_t launch_gemm_tc(llx_session* s, const Binding& bd, int in, const LinearArgs& a, bool gated) {
  llx_model* m = s->m;
  const int R = a.R, N = a.N, K = a.K;
  int nt = 16, ks = 1;
  pick_tc_tiling(R, N, K, m->sms, &nt, &ks);
  if (gated && nt < 32) {
    nt = 32;
    ks = 1;
  }
  const int row_tiles = (R + 127) / 128;
  // small decode batches (R <= 32): the swapped-operand kernel (128 channels x up to 32 rows
  // per tile), K split over a cluster so that about one CTA per SM streams the weights.  Its
  // split-K partial tile is [128][NB] int32, summed over DSMEM; above 32 rows that exchange
  // costs more than the row-tile kernel's, which wins from 64 rows up (measured at C3).
  if (R <= 32 && m->opts.gemm_path != 4) {
    const int ch_tiles = (N + 127) / 128;
    const int nkb = (K + 127) / 128;
    int kss = (m->sms + ch_tiles / 2) / ch_tiles;
    kss = std::max(1, std::min({kss, nkb, 8}));
    const bool persistent = (N + 255) / 256 >= 2 * m->sms;
    if (!persistent) {
      const int nb = sab_rows_per_tile(R);
      const CUtensorMap& mab = tmap(s, a.A, (int64_t)bd.rows[in], K, nb);
      const CUtensorMap& mwb = tmap(s, a.W, N, K, 128);
      return launch_linear_sab(mab, mwb, a, nb, kss, s->d_fault, s->st);
    }
  }
  const CUtensorMap& ma = tmap(s, a.A, (int64_t)bd.rows[in], K, 128);
  if (ks == 1) {
    for (int pnt : {256, 128}) {
      if ((N + pnt - 1) / pnt * row_tiles >= 2 * m->sms) {
        const CUtensorMap& mw = tmap(s, a.W, N, K, pnt);
        return launch_linear_tc_persistent(ma, mw, a, pnt, m->sms, s->d_fault, s->st);
      }
    }
  }
  const CUtensorMap& mw = tmap(s, a.W, N, K, nt);
  return launch_linear_tc(ma, mw, a, nt, ks, s->d_fault, s->st);
}

static int enqueue_steps(llx_session* s, const Binding& bd, size_t from, size_t to, int R, int M) {
  int launches = 0;
  for (size_t i = from; i < to; ++i) launches += enqueue_one(s, bd, s->m->steps[i], R, M);
  return launches;
}

// GEMM path of a linear step over R rows: 3 = tensor cores (4: tensor cores without the
// swapped-operand decode kernel, a cross-check), else a CUDA-core schedule
static int gemm_path_for(const llx_model* m, int R) {
  int path = m->opts.gemm_path;
  if (path == 4) return 3;
  if (path == 0) path = R >= 16 ? 3 : 1;
  return path;
}

// The model output is a plain linear on the tensor-core path: its epilogue produced the
// argmax keys, which only need decoding; otherwise a full argmax pass over the logits runs.
static bool output_argmax_fused(const llx_model* m, int R) {
  for (const Step& x : m->steps)
    if (x.kind == SK::Linear && x.out == m->output_act) return gemm_path_for(m, R) == 3;
  return false;
}

// channels of this rank's output that are real vocabulary entries (all of them on one GPU)
static int local_vocab(const llx_model* m) {
  return std::max(0, std::min(m->vocab_padded, m->vocab - m->vocab_base));
}

static void tp_check(bool ok, const std::string& err) {
  if (!ok) throw Error(LLX_ERR_CUDA, err);
}

// argmax tokens of R output rows into d_argmax.  Under tensor parallelism every rank holds
// packed keys of its vocabulary shard (global indices); a uint64 max all-reduce picks the
// global first maximum before the keys are decoded.
static void launch_output_argmax(llx_session* s, const void* logits, int R) {
  const llx_model* m = s->m;
  const bool fused = output_argmax_fused(m, R);
  cudaError_t e = cudaSuccess;
  // keys were zeroed by the launch's embed step (or by llx_run_rows)
  if (!fused)
    e = launch_argmax((const int16_t*)logits, R, m->vocab_padded, local_vocab(m), m->vocab_base, s->d_amax_key,
                      s->st);
  if (e == cudaSuccess && m->tp) {
    std::string err;
    tp_check(tp_allreduce_max_u64(m->tp, s->d_amax_key, R, s->st, &err), err);
  }
  if (e == cudaSuccess) e = launch_amax_finish(s->d_amax_key, s->d_argmax, R, s->st);
  if (e != cudaSuccess) throw Error(LLX_ERR_CUDA, std::string("argmax launch failed: ") + cudaGetErrorString(e));
}

static int enqueue_one(llx_session* s, const Binding& bd, const Step& x, int R, int M) {
  llx_model* m = s->m;
  cudaStream_t st = s->st;
  // a plan step (not a constituent of a fused one): an RMSNorm the next GEMV runs in its
  // prologue launches nothing; that GEMV gets the norm's parameters
  const Step* steps0 = m->steps.data();
  const bool top = &x >= steps0 && &x < steps0 + m->steps.size();
  const size_t idx = top ? (size_t)(&x - steps0) : 0;
  if (top && norm_folds_into_next(s, idx, R)) return 0;
  const Step* fold = top && idx > 0 && norm_folds_into_next(s, idx - 1, R) ? &m->steps[idx - 1] : nullptr;
  auto P = [&](int a) { return a < 0 ? nullptr : bd.p[a]; };
  // the folded RMSNorm's row and parameters for the GEMV prologue
  auto apply_fold = [&](LinearArgs& a) {
    if (!fold) return;
    a.nx = (const int16_t*)P(fold->in);
    a.ngamma = (const int16_t*)dptr(m, fold->gamma_off);
    a.n_eps = fold->eps_t;
    a.n_C = fold->C;
    a.n_sh = fold->sh_post;
    a.n_Mq = fold->Mq;
    a.n_Sq = fold->Sq;
  };
  // an output that no later step reads (and no dump keeps) is not stored
  auto Pused = [&](int a) { return (a < 0 || (!s->keep && m->act_uses[a] == 0)) ? nullptr : bd.p[a]; };
  {
    cudaError_t e = cudaSuccess;
    switch (x.kind) {
      case SK::Embed:
        e = launch_embed(s->d_tokens, (const int16_t*)dptr(m, m->embed_off), (int16_t*)P(x.out), R, m->dim,
                         m->vocab, s->d_err, s->d_amax_key, st);
        break;
      case SK::RmsNorm:
        e = launch_rmsnorm((const int16_t*)P(x.in), (const int16_t*)dptr(m, x.gamma_off),
                           (int16_t*)(x.out2 >= 0 ? Pused(x.out) : P(x.out)), (int8_t*)P(x.out2), R * x.heads, x.K, x.eps_t, x.C, x.sh_post, x.Mq, x.Sq, st);
        break;
      case SK::Quant:
        e = launch_quant((const int16_t*)P(x.in), (int8_t*)P(x.out), (int64_t)R * m->acts[x.in].cols, x.Mq, x.Sq, st);
        break;
      case SK::Linear: {
        LinearArgs a{};
        a.A = (const int8_t*)P(x.in);
        a.W = (const int8_t*)dptr(m, x.w_off);
        a.bias = (const int32_t*)dptr(m, x.bias_off);
        a.rq = (const int32_t*)dptr(m, x.rq_off);
        a.aux = (const int16_t*)P(x.in2);
        a.out = P(x.out);
        a.R = R;
        a.N = x.N;
        a.K = x.K;
        a.out_i8 = x.out_i8;
        a.epi = x.epi;
        a.silu_Mi = x.silu_Mi;
        a.silu_Si = x.silu_Si;
        a.silu_sh = x.silu_sh;
        a.aux_shift = x.aux_shift;
        a.luts = m->d_luts;
        a.narrow = x.narrow;
        const int path = gemm_path_for(m, R);
        if (path == 3 && x.out == m->output_act) {
          a.amax_key = s->d_amax_key;
          a.amax_vocab = local_vocab(m);
          a.amax_base = m->vocab_base;
          // argmax-only launches skip the logits store: nothing reads them
          if (!s->store_logits) a.out = nullptr;
        }
        apply_fold(a);
        if (path == 3)
          e = launch_gemm_tc(s, bd, x.in, a, false);
        else
          e = launch_linear(a, path, st);
        break;
      }
      case SK::LinearPartial: {
        LinearArgs a{};
        a.A = (const int8_t*)P(x.in);
        a.W = (const int8_t*)dptr(m, x.w_off);
        a.out = P(x.out);
        a.R = R;
        a.N = x.N;
        a.K = x.K;
        a.out_i32 = 1;
        a.luts = m->d_luts;
        const int path = gemm_path_for(m, R);
        if (path == 3)
          e = launch_gemm_tc(s, bd, x.in, a, false);
        else
          e = launch_linear(a, path, st);
        break;
      }
      case SK::AllReduce: {
        if (!m->tp) return 0;  // a one-rank group: the partial sums are already complete
        std::string err;
        tp_check(tp_allreduce_sum_i32(m->tp, (int32_t*)P(x.in), (size_t)R * x.N, st, &err), err);
        return 1;
      }
      case SK::Requant: {
        LinearArgs a{};
        a.bias = (const int32_t*)dptr(m, x.bias_off);
        a.rq = (const int32_t*)dptr(m, x.rq_off);
        a.aux = (const int16_t*)P(x.in2);
        a.out = P(x.out);
        a.R = R;
        a.N = x.N;
        a.out_i8 = x.out_i8;
        a.epi = x.epi;
        a.silu_Mi = x.silu_Mi;
        a.silu_Si = x.silu_Si;
        a.silu_sh = x.silu_sh;
        a.aux_shift = x.aux_shift;
        a.luts = m->d_luts;
        e = launch_requant((const int32_t*)P(x.in), a, st);
        break;
      }
      case SK::Rope: {
        int8_t* kc = x.write_k ? s->kv_layer.at(x.layer).first : nullptr;
        e = launch_rope((const int16_t*)P(x.in), (int16_t*)(x.out2 >= 0 ? Pused(x.out) : P(x.out)), (int8_t*)P(x.out2),
                        x.Mq, x.Sq, kc, R, M, x.H,
                        x.D, (const int16_t*)dptr(m, m->cos_off), (const int16_t*)dptr(m, m->sin_off), s->d_pos,
                        m->max_seq, st);
        break;
      }
      case SK::KvWrite: {
        auto kv = s->kv_layer.at(x.layer);
        e = launch_kv_write((const int8_t*)P(x.in), (const int8_t*)P(x.in2), kv.first, kv.second, R, M, x.Hkv, x.D,
                            s->d_pos, m->max_seq, st);
        break;
      }
      case SK::Attention: {
        auto kv = s->kv_layer.at(x.layer);
        AttnArgs a{};
        a.q = (const int8_t*)P(x.in);
        a.kc = kv.first;
        a.vc = kv.second;
        a.out = (int8_t*)P(x.out);
        a.B = R / M;
        a.M = M;
        a.H = x.H;
        a.Hkv = x.Hkv;
        a.D = x.D;
        a.max_seq = m->max_seq;
        a.d_pos = s->d_pos;
        a.Ms = x.Ms;
        a.Ss = x.Ss;
        a.Mo = x.Mo;
        a.So = x.So;
        a.prob_bits = x.prob_bits;
        a.luts = m->d_luts;
        a.err = s->d_fault;
        if (M == 1 && x.rope_step >= 0 && !s->keep) {
          const Step& rg = m->steps[x.rope_step];
          const Step& q = rg.parts[0];
          const Step& k = rg.parts[1];
          const Step& v = rg.parts[2];
          a.rq16 = (const int16_t*)P(q.in);
          a.rk16 = (const int16_t*)P(k.in);
          a.rv8 = (const int8_t*)P(v.in2);
          a.kc_out = kv.first;
          a.vc_out = kv.second;
          a.cos_tab = (const int16_t*)dptr(m, m->cos_off);
          a.sin_tab = (const int16_t*)dptr(m, m->sin_off);
          a.q_M = q.Mq;
          a.q_S = q.Sq;
          a.k_M = k.Mq;
          a.k_S = k.Sq;
        }
        e = launch_attention(a, st);
        break;
      }
      case SK::LinearGroup:
      case SK::Gated: {
        const int path = gemm_path_for(m, R);
        if (path == 2) {
          // the tiled CUDA-core schedule runs the constituent ops one by one
          int n = 0;
          for (const Step& p : x.parts) n += enqueue_one(s, bd, p, R, M);
          return n;
        }
        LinearArgs a{};
        a.A = (const int8_t*)P(x.in);
        a.W = (const int8_t*)dptr(m, x.w_off);
        a.bias = (const int32_t*)dptr(m, x.bias_off);
        a.rq = (const int32_t*)dptr(m, x.rq_off);
        a.R = R;
        a.N = x.N;
        a.K = x.K;
        a.luts = m->d_luts;
        a.narrow = x.narrow;
        if (x.kind == SK::LinearGroup) {
          a.nseg = x.nseg;
          for (int i = 0; i <= x.nseg; ++i) a.seg_start[i] = x.seg_start[i];
          for (int i = 0; i < x.nseg; ++i) {
            a.seg_out[i] = P(x.parts[i].out);
            a.seg_i8[i] = x.parts[i].out_i8;
          }
        } else {
          const Step& g = x.parts[0];
          const Step& u = x.parts[1];
          a.gated = 1;
          a.Nout = u.N;
          a.silu_Mi = g.silu_Mi;
          a.silu_Si = g.silu_Si;
          a.silu_sh = g.silu_sh;
          a.aux_shift = u.aux_shift;
          a.g_out = (int16_t*)Pused(g.out);
          a.f_out = (int16_t*)(x.parts.size() > 2 ? Pused(u.out) : P(u.out));
          if (x.parts.size() > 2) {
            a.q_out = (int8_t*)P(x.parts[2].out);
            a.q_M = x.parts[2].Mq;
            a.q_S = x.parts[2].Sq;
          }
        }
        // tensor cores, or (few rows) the GEMV, which fuses the group / pair the same way
        apply_fold(a);
        e = path == 3 ? launch_gemm_tc(s, bd, x.in, a, x.kind == SK::Gated) : launch_linear(a, 1, st);
        break;
      }
      case SK::RopeGroup: {
        if (M == 1 && x.folded && !s->keep) return 0;  // done by the decode attention
        const Step& q = x.parts[0];
        const Step& k = x.parts[1];
        const Step& v = x.parts[2];
        auto kv = s->kv_layer.at(k.layer);
        RopeJob jq{(const int16_t*)P(q.in), (int16_t*)Pused(q.out), (int8_t*)P(q.out2), q.Mq, q.Sq, nullptr, q.H};
        RopeJob jk{(const int16_t*)P(k.in), (int16_t*)Pused(k.out), (int8_t*)P(k.out2), k.Mq, k.Sq, kv.first, k.H};
        e = launch_rope_group(jq, jk, (const int8_t*)P(v.in2), s->kv_layer.at(v.layer).second, v.Hkv, R, M, q.D,
                              (const int16_t*)dptr(m, m->cos_off), (const int16_t*)dptr(m, m->sin_off), s->d_pos,
                              m->max_seq, st);
        break;
      }
      case SK::Add:
        e = launch_add((const int16_t*)P(x.in), (const int16_t*)P(x.in2), (int16_t*)P(x.out),
                       (int64_t)R * m->acts[x.in].cols, x.sh, st);
        break;
      case SK::Mul:
        e = launch_mul((const int16_t*)P(x.in), (const int16_t*)P(x.in2), (int16_t*)P(x.out),
                       (int64_t)R * m->acts[x.in].cols, x.sh, st);
        break;
      case SK::Silu:
        e = launch_silu((const int16_t*)P(x.in), (int16_t*)P(x.out), (int64_t)R * m->acts[x.in].cols, x.silu_Mi,
                        x.silu_Si, x.silu_sh, m->d_luts, st);
        break;
    }
    if (e != cudaSuccess) throw Error(LLX_ERR_CUDA, "launch of step '" + x.label + "' failed: " + cudaGetErrorString(e));
  }
  return 1;
}

// ---- activation arena: first-fit reuse by liveness over the step list -------------------------
struct ArenaPlanner {
  std::map<size_t, size_t> holes;  // offset -> size
  size_t top = 0, peak = 0;
  size_t alloc(size_t n) {
    for (auto it = holes.begin(); it != holes.end(); ++it) {
      if (it->second >= n) {
        const size_t off = it->first, rest = it->second - n;
        holes.erase(it);
        if (rest) holes[off + n] = rest;
        return off;
      }
    }
    const size_t off = top;
    top += n;
    peak = std::max(peak, top);
    return off;
  }
  void release(size_t off, size_t n) {
    auto it = holes.emplace(off, n).first;
    auto nx = std::next(it);
    if (nx != holes.end() && it->first + it->second == nx->first) {
      it->second += nx->second;
      holes.erase(nx);
    }
    if (it != holes.begin()) {
      auto pv = std::prev(it);
      if (pv->first + pv->second == it->first) {
        pv->second += it->second;
        holes.erase(it);
        it = pv;
      }
    }
    if (it->first + it->second == top) {
      top = it->first;
      holes.erase(it);
    }
  }
};

static size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

static void plan_arena(llx_session* s) {
  llx_model* m = s->m;
  const size_t rows = (size_t)s->B * s->max_rows;
  const size_t tail_rows = (size_t)s->B * s->max_tail_rows;
  const size_t na = m->acts.size();
  std::vector<char> in_tail(na, 0);
  for (size_t i = m->tail_start; i < m->steps.size(); ++i)
    for (int a : step_outs(m->steps[i])) in_tail[a] = 1;
  std::vector<size_t> bytes(na);
  s->act_rows.assign(na, 0);
  s->tail_rows_alloc = tail_rows;
  for (size_t i = 0; i < na; ++i) {
    s->act_rows[i] = in_tail[i] ? tail_rows : rows;
    bytes[i] = round256(s->act_rows[i] * m->acts[i].cols * m->acts[i].elem);
  }
  s->act_off.assign(na, 0);
  ArenaPlanner ap;
  if (s->keep) {
    for (size_t i = 0; i < na; ++i) s->act_off[i] = ap.alloc(bytes[i]);
  } else {
    const int ns = (int)m->steps.size();
    std::vector<int> def(na, ns), last(na, -1);
    for (int i = 0; i < ns; ++i) {
      const Step& x = m->steps[i];
      for (int a : step_outs(x)) def[a] = std::min(def[a], i);
      for (int a : step_ins(x)) last[a] = std::max(last[a], i);
    }
    last[m->output_act] = ns;
    // a decode attention with its RoPE group folded in reads that group's inputs (q and k
    // before rotation, v): they live through the attention step, so its output never
    // takes their memory while other CTAs still read them
    for (int i = 0; i < ns; ++i) {
      const Step& x = m->steps[i];
      if (x.kind != SK::Attention || x.rope_step < 0) continue;
      for (int a : step_ins(m->steps[x.rope_step])) last[a] = std::max(last[a], i);
    }
    // a norm folded into the next GEMV's prologue is read by that GEMV: its input lives
    // through it, so the GEMV's output never takes the row other blocks are still reading
    for (int i = 0; i + 1 < ns; ++i)
      if (norm_pair(m, (size_t)i)) last[m->steps[i].in] = std::max(last[m->steps[i].in], i + 1);
    for (size_t a = 0; a < na; ++a) last[a] = std::max(last[a], def[a]);
    for (int i = 0; i <= ns; ++i) {
      for (size_t a = 0; a < na; ++a)
        if (def[a] == i) s->act_off[a] = ap.alloc(bytes[a]);
      for (size_t a = 0; a < na; ++a)
        if (last[a] == i && def[a] <= i) ap.release(s->act_off[a], bytes[a]);
    }
  }
  size_t extra = ap.peak;
  s->tail_off.clear();
  for (int a : m->tail_inputs) {
    s->tail_off.push_back(extra);
    extra += round256(tail_rows * m->acts[a].cols * m->acts[a].elem);
  }
  s->arena_bytes = std::max<size_t>(extra, 256);
}

__global__ void k_decode_finalize(const int32_t* argmax, int32_t* tokens,
                                  int32_t* hist, int32_t* pos, int32_t* step, int B, int cap) {
  pdl_trigger();
  pdl_wait();
  __shared__ int s_step;
  if (threadIdx.x == 0) s_step = *step;
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int32_t t = argmax[b];
    tokens[b] = t;
    if (s_step < cap) hist[(int64_t)s_step * B + b] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *pos += 1;
    *step = s_step + 1;
  }
}

static void ensure_i16(llx_session* s, size_t n) {
  if (s->h_i16_n >= n) return;
  LLX_CUDA(cudaStreamSynchronize(s->st));
  if (s->h_i16) cudaFreeHost(s->h_i16);
  s->h_i16 = nullptr;
  LLX_CUDA(cudaMallocHost(&s->h_i16, n * sizeof(int16_t)));
  s->h_i16_n = n;
}

static void check_device_error(llx_session* s) {
  int32_t err[2] = {0, 0};
  LLX_CUDA(cudaMemcpyAsync(err, s->d_err, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, s->st));
  LLX_CUDA(cudaStreamSynchronize(s->st));
  if (err[0] || err[1]) {
    LLX_CUDA(cudaMemsetAsync(s->d_err, 0, 2 * sizeof(int32_t), s->st));
    LLX_CUDA(cudaStreamSynchronize(s->st));
    if (err[1])
      throw Error(LLX_ERR_DEVICE, "a tensor-core pipeline wait timed out (code " + std::to_string(err[1]) + ")");
    throw Error(LLX_ERR_RANGE, "token ID exceeds model vocabulary");
  }
}

// POS and the step counter go through their own pinned words; the stream is drained
// first so the host never rewrites a word a pending copy still reads.
static void set_pos(llx_session* s, int pos) {
  LLX_CUDA(cudaStreamSynchronize(s->st));
  s->h_pos[0] = pos;
  s->h_pos[1] = 0;
  LLX_CUDA(cudaMemcpyAsync(s->d_pos, s->h_pos, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, s->st));
}

// Launch over M rows per sequence at pos; input rows already in the input buffer (or
// tokens in d_tokens when with_embed). rec: host [B][n_rec] or null (all rows).
static void run_launch(llx_session* s, int M, int pos, bool with_embed, const int32_t* rec, int n_rec) {
  llx_model* m = s->m;
  const int R = s->B * M;
  set_pos(s, pos);
  bool tail = false;
  if (rec) {
    for (int b = 0; b < s->B && !tail; ++b)
      for (int j = 0; j < n_rec; ++j)
        if (n_rec != M || rec[(size_t)b * n_rec + j] != j) {
          tail = true;
          break;
        }
  }
  Binding bd = bind(s, false);
  const size_t first = with_embed ? 0 : 1;
  int Rtail = R;
  if (!tail) {
    require(M <= s->max_tail_rows, LLX_ERR_RANGE,
            "a launch records at most " + std::to_string(s->max_tail_rows) + " rows per sequence");
    enqueue_steps(s, bd, first, m->steps.size(), R, M);
  } else {
    require(n_rec <= s->max_tail_rows, LLX_ERR_RANGE,
            "a launch records at most " + std::to_string(s->max_tail_rows) + " rows per sequence");
    Rtail = s->B * n_rec;
    for (int b = 0; b < s->B; ++b)
      for (int j = 0; j < n_rec; ++j) s->h_rec[(size_t)b * n_rec + j] = b * M + rec[(size_t)b * n_rec + j];
    LLX_CUDA(cudaMemcpyAsync(s->d_rec, s->h_rec, sizeof(int32_t) * Rtail, cudaMemcpyHostToDevice, s->st));
    enqueue_steps(s, bd, first, m->tail_start, R, M);
    Binding bt = bd;
    for (size_t t = 0; t < m->tail_inputs.size(); ++t) {
      const int a = m->tail_inputs[t];
      void* dst = s->arena + s->tail_off[t];
      const cudaError_t e =
          launch_gather_rows(bd.p[a], dst, s->d_rec, Rtail, m->acts[a].cols * m->acts[a].elem, s->st);
      if (e != cudaSuccess) throw Error(LLX_ERR_CUDA, cudaGetErrorString(e));
      bt.p[a] = dst;
      bt.rows[a] = s->tail_rows_alloc;
    }
    enqueue_steps(s, bt, m->tail_start, m->steps.size(), Rtail, n_rec);
  }
  launch_output_argmax(s, bd.p[m->output_act], Rtail);
  s->last_R = R;
  s->last_Rtail = Rtail;
  s->last_tail = tail;
  s->last_logits = true;
}

// logits of the last launch's first `rows` output rows -> host [rows][vocab_padded_full].
// Under tensor parallelism the ranks' vocabulary shards are all-gathered first (a
// collective: every rank of the group makes the same call).
static void fetch_logits(llx_session* s, int rows, int16_t* host) {
  llx_model* m = s->m;
  const Binding bd = bind(s, false);
  const size_t vl = m->vocab_padded;
  if (!m->tp) {
    ensure_i16(s, (size_t)rows * vl);
    LLX_CUDA(cudaMemcpyAsync(s->h_i16, bd.p[m->output_act], sizeof(int16_t) * rows * vl, cudaMemcpyDeviceToHost,
                             s->st));
    LLX_CUDA(cudaStreamSynchronize(s->st));
    std::memcpy(host, s->h_i16, sizeof(int16_t) * rows * vl);
    return;
  }
  const size_t W = m->tp_world, n = W * rows * vl;
  if (s->gather_n < n) {
    LLX_CUDA(cudaStreamSynchronize(s->st));
    if (s->d_gather) cudaFree(s->d_gather);
    s->d_gather = nullptr;
    s->gather_n = 0;
    LLX_CUDA(cudaMalloc(&s->d_gather, n * sizeof(int16_t)));
    s->gather_n = n;
  }
  ensure_i16(s, n);
  std::string err;
  tp_check(tp_allgather_bytes(m->tp, bd.p[m->output_act], s->d_gather, sizeof(int16_t) * rows * vl, s->st, &err), err);
  LLX_CUDA(cudaMemcpyAsync(s->h_i16, s->d_gather, sizeof(int16_t) * n, cudaMemcpyDeviceToHost, s->st));
  LLX_CUDA(cudaStreamSynchronize(s->st));
  const size_t full = m->vocab_padded_full;
  for (size_t r = 0; r < (size_t)rows; ++r)
    for (size_t w = 0; w < W; ++w)
      std::memcpy(host + r * full + w * vl, s->h_i16 + (w * rows + r) * vl, sizeof(int16_t) * vl);
}

static void copy_outputs(llx_session* s, int rows, int16_t* logits, int32_t* argmax) {
  if (argmax)
    LLX_CUDA(cudaMemcpyAsync(s->h_am, s->d_argmax, sizeof(int32_t) * rows, cudaMemcpyDeviceToHost, s->st));
  LLX_CUDA(cudaStreamSynchronize(s->st));
  if (argmax) std::memcpy(argmax, s->h_am, sizeof(int32_t) * rows);
  if (logits) fetch_logits(s, rows, logits);
}

static void stage_tokens(llx_session* s, const int32_t* tokens, int n) {
  for (int i = 0; i < n; ++i)
    require(tokens[i] < s->m->vocab, LLX_ERR_RANGE, "token ID exceeds model vocabulary");
  LLX_CUDA(cudaStreamSynchronize(s->st));
  std::memcpy(s->h_tok, tokens, sizeof(int32_t) * n);
  LLX_CUDA(cudaMemcpyAsync(s->d_tokens, s->h_tok, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s->st));
}

// The M = 1 decode step as a CUDA graph; with_logits selects the variant whose output
// linear also stores the logits rows (otherwise only the fused argmax keys are produced).
static cudaGraphExec_t build_decode_graph(llx_session* s, bool with_logits) {
  cudaGraphExec_t& exec = s->decode_exec[with_logits ? 1 : 0];
  if (exec) return exec;
  llx_model* m = s->m;
  Binding bd = bind(s, false);
  LLX_CUDA(cudaStreamSynchronize(s->st));
  cudaGraph_t graph;
  LLX_CUDA(cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal));
  int n = 0;
  s->store_logits = with_logits;
  try {
    n = enqueue_steps(s, bd, 0, m->steps.size(), s->B, 1);
    launch_output_argmax(s, bd.p[m->output_act], s->B);
    LLX_CUDA(launch_k(k_decode_finalize, dim3(1), dim3(256), 0, s->st, (const int32_t*)s->d_argmax, s->d_tokens,
                      s->d_hist, s->d_pos, s->d_step, s->B, s->hist_cap));
  } catch (...) {
    s->store_logits = true;
    cudaStreamEndCapture(s->st, &graph);
    throw;
  }
  s->store_logits = true;
  LLX_CUDA(cudaStreamEndCapture(s->st, &graph));
  const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  LLX_CUDA(e);
  s->decode_launches = n + 2;
  return exec;
}

static void session_create(llx_model* m, int batch, int max_rows, int keep, llx_session* s) {
  require(batch >= 1, LLX_ERR_INVALID, "batch must be >= 1");
  if (m->tp_world > 1) {
    require(m->tp != nullptr, LLX_ERR_INVALID, "tensor-parallel rank graph: call llx_tp_init before creating a session");
    // collectives of two sessions on one communicator could interleave differently per rank
    require(m->n_sessions == 0, LLX_ERR_UNSUPPORTED, "a tensor-parallel model serves one session at a time");
  }
  require(max_rows >= 1 && max_rows <= m->max_seq, LLX_ERR_INVALID, "max_rows must be in [1, max_seq]");
  s->m = m;
  m->n_sessions++;
  s->B = batch;
  s->max_rows = max_rows;
  s->keep = keep != 0;
  // the row-independent tail (final norm, lm_head, ...) holds every row of a launch when
  // that costs at most 2 GB of logits, else 64 recorded rows per sequence
  s->max_tail_rows = (double)batch * max_rows * m->vocab_padded * 2.0 <= 2.0e9 ? max_rows : std::min(max_rows, 64);
  LLX_CUDA(cudaSetDevice(m->device));
  LLX_CUDA(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
  plan_arena(s);
  LLX_CUDA(cudaMalloc(&s->arena, s->arena_bytes));
  LLX_CUDA(cudaMemset(s->arena, 0, s->arena_bytes));
  size_t kvb = 0;
  for (auto& kv : m->kv_layers) kvb += 2 * (size_t)batch * kv.second.Hkv * m->max_seq * kv.second.D;
  s->kv_bytes = std::max<size_t>(kvb, 256);
  LLX_CUDA(cudaMalloc(&s->kv, s->kv_bytes));
  LLX_CUDA(cudaMemset(s->kv, 0, s->kv_bytes));
  size_t off = 0;
  for (auto& kv : m->kv_layers) {
    const size_t one = (size_t)batch * kv.second.Hkv * m->max_seq * kv.second.D;
    s->kv_layer[kv.first] = {s->kv + off, s->kv + off + one};
    off += 2 * one;
  }
  const size_t rows = (size_t)batch * max_rows;
  s->hist_cap = m->max_seq;
  LLX_CUDA(cudaMalloc(&s->d_tokens, sizeof(int32_t) * rows));
  LLX_CUDA(cudaMalloc(&s->d_rec, sizeof(int32_t) * rows));
  LLX_CUDA(cudaMalloc(&s->d_argmax, sizeof(int32_t) * rows));
  LLX_CUDA(cudaMalloc(&s->d_amax_key, sizeof(unsigned long long) * rows));
  LLX_CUDA(cudaMemset(s->d_amax_key, 0, sizeof(unsigned long long) * rows));
  LLX_CUDA(cudaMalloc(&s->d_hist, sizeof(int32_t) * (size_t)s->hist_cap * batch));
  LLX_CUDA(cudaMalloc(&s->d_pos, sizeof(int32_t) * 4));
  s->d_step = s->d_pos + 1;
  s->d_err = s->d_pos + 2;
  s->d_fault = s->d_pos + 3;
  LLX_CUDA(cudaMemset(s->d_pos, 0, sizeof(int32_t) * 4));
  LLX_CUDA(cudaMemset(s->d_tokens, 0, sizeof(int32_t) * rows));
  LLX_CUDA(cudaMallocHost(&s->h_tok, sizeof(int32_t) * rows));
  LLX_CUDA(cudaMallocHost(&s->h_rec, sizeof(int32_t) * rows));
  LLX_CUDA(cudaMallocHost(&s->h_am, sizeof(int32_t) * rows));
  LLX_CUDA(cudaMallocHost(&s->h_pos, sizeof(int32_t) * 4));
  // the clears above run on the legacy default stream, which the session's non-blocking
  // stream does not wait for, and cudaMemset of device memory may return before it is
  // done: finish them before any launch (or peer) can touch these buffers
  LLX_CUDA(cudaDeviceSynchronize());
}

static void session_free(llx_session* s) {
  if (!s) return;
  if (s->m) {
    cudaSetDevice(s->m->device);
    s->m->n_sessions--;
  }
  if (s->st) cudaStreamSynchronize(s->st);
  for (cudaGraphExec_t g : s->decode_exec)
    if (g) cudaGraphExecDestroy(g);
  for (void* p : {(void*)s->arena, (void*)s->kv, (void*)s->d_tokens, (void*)s->d_rec, (void*)s->d_argmax,
                  (void*)s->d_hist, (void*)s->d_pos, (void*)s->d_amax_key, (void*)s->d_gather, (void*)s->d_flush})
    if (p) cudaFree(p);
  for (void* p : {(void*)s->h_tok, (void*)s->h_rec, (void*)s->h_am, (void*)s->h_pos, (void*)s->h_i16})
    if (p) cudaFreeHost(p);
  if (s->st) cudaStreamDestroy(s->st);
}

static void reset_kv(llx_session* s) {
  LLX_CUDA(cudaMemsetAsync(s->kv, 0, s->kv_bytes, s->st));
  LLX_CUDA(cudaStreamSynchronize(s->st));
}

}  // namespace llx

// ---------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------
using namespace llx;

template <class F>
static llx_status guarded(F&& f) {
  try {
    f();
    return LLX_OK;
  } catch (const Error& e) {
    g_err = e.what();
    return e.code;
  } catch (const std::bad_alloc&) {
    g_err = "host allocation failed";
    return LLX_ERR_OOM;
  } catch (const std::exception& e) {
    g_err = e.what();
    return LLX_ERR_INVALID;
  }
}

extern "C" {

const char* llx_last_error(void) { return g_err.c_str(); }
const char* llx_version(void) { return "llx 0.1 sm_100a"; }

llx_status llx_binary_version(int device, int* version) {
  return guarded([&] {
    require(version != nullptr, LLX_ERR_INVALID, "null argument");
    LLX_CUDA(cudaSetDevice(device));
    cudaFuncAttributes fa{};
    LLX_CUDA(cudaFuncGetAttributes(&fa, k_decode_finalize));
    *version = fa.binaryVersion;
  });
}

llx_status llx_model_load(const char* dir, const llx_opts* opts, llx_model** out) {
  return guarded([&] {
    require(dir && out, LLX_ERR_INVALID, "null argument");
    auto m = std::make_unique<llx_model>();
    m->opts.device = 0;
    m->opts.fuse = 1;
    m->opts.gemm_path = 0;
    m->opts.pdl = 1;
    if (opts) m->opts = *opts;
    g_pdl = m->opts.pdl;
    m->device = m->opts.device;
    int ndev = 0;
    LLX_CUDA(cudaGetDeviceCount(&ndev));
    require(m->device >= 0 && m->device < ndev, LLX_ERR_INVALID, "no such CUDA device");
    try {
      load_model(m.get(), dir);
    } catch (...) {
      if (m->d_blob) cudaFree(m->d_blob);
      if (m->d_luts) cudaFree(m->d_luts);
      throw;
    }
    *out = m.release();
  });
}

void llx_model_destroy(llx_model* m) {
  if (!m) return;
  tp_comm_destroy(m->tp);
  cudaSetDevice(m->device);
  if (m->d_blob) cudaFree(m->d_blob);
  if (m->d_luts) cudaFree(m->d_luts);
  delete m;
}

llx_status llx_model_get_info(const llx_model* m, llx_model_info* o) {
  return guarded([&] {
    require(m && o, LLX_ERR_INVALID, "null argument");
    o->dim = m->dim;
    o->n_layers = m->n_layers;
    o->n_heads = m->n_heads;
    o->n_kv_heads = m->n_kv_heads;
    o->head_dim = m->head_dim;
    o->ffn = m->ffn;
    o->vocab = m->vocab;
    o->max_seq = m->max_seq;
    o->prefill_m = m->prefill_m;
    o->E_RES = m->E_RES;
    o->E_LOGIT = m->E_LOGIT;
    o->n_ops = m->n_ops;
    o->n_steps = (int)m->steps.size();
    o->n_activations = (int)m->acts.size();
    o->weight_bytes = m->blob_bytes;
    o->vocab_padded = m->vocab_padded_full;
    o->tp_world = m->tp_world;
    o->tp_rank = m->tp_rank;
    o->vocab_base = m->vocab_base;
    o->vocab_local = m->vocab_padded;
  });
}

llx_status llx_tp_unique_id(void* id) {
  return guarded([&] {
    require(id, LLX_ERR_INVALID, "null argument");
    std::string err;
    require(tp_unique_id(id, &err), LLX_ERR_CUDA, err);
  });
}

llx_status llx_tp_init(llx_model* m, const void* id, int rank, int world) {
  return guarded([&] {
    require(m && id, LLX_ERR_INVALID, "null argument");
    require(m->tp == nullptr, LLX_ERR_INVALID, "llx_tp_init: the model already has a communicator");
    require(m->n_sessions == 0, LLX_ERR_INVALID, "llx_tp_init: call it before creating sessions");
    require(world == m->tp_world && rank == m->tp_rank, LLX_ERR_INVALID,
            "llx_tp_init: rank " + std::to_string(rank) + " of " + std::to_string(world) +
                " does not match the graph's model.tp (rank " + std::to_string(m->tp_rank) + " of " +
                std::to_string(m->tp_world) + ")");
    std::string err;
    TpComm* c = tp_comm_create(id, rank, world, m->device, &err);
    require(c != nullptr, LLX_ERR_CUDA, err);
    m->tp = c;
  });
}

llx_status llx_session_create(llx_model* m, int batch, int max_rows, int keep_acts, llx_session** out) {
  return guarded([&] {
    require(m && out, LLX_ERR_INVALID, "null argument");
    auto s = std::make_unique<llx_session>();
    try {
      session_create(m, batch, max_rows, keep_acts, s.get());
    } catch (...) {
      session_free(s.get());
      throw;
    }
    *out = s.release();
  });
}

void llx_session_destroy(llx_session* s) {
  session_free(s);
  delete s;
}

llx_status llx_session_reset(llx_session* s) {
  return guarded([&] {
    require(s, LLX_ERR_INVALID, "null session");
    reset_kv(s);
  });
}

llx_status llx_run(llx_session* s, const int32_t* tokens, int M, int pos, const int32_t* rec_rows, int n_rec,
                   int16_t* logits, int32_t* argmax) {
  return guarded([&] {
    require(s && tokens, LLX_ERR_INVALID, "null argument");
    require(M >= 1 && M <= s->max_rows, LLX_ERR_RANGE, "M outside [1, max_rows]");
    require(pos >= 0 && pos + M <= s->m->max_seq, LLX_ERR_RANGE,
            "positions " + std::to_string(pos) + ".." + std::to_string(pos + M - 1) +
                " exceed max_seq=" + std::to_string(s->m->max_seq));
    if (rec_rows) {
      require(n_rec >= 1 && n_rec <= M, LLX_ERR_RANGE, "n_rec outside [1, M]");
      for (int i = 0; i < s->B * n_rec; ++i)
        require(rec_rows[i] >= 0 && rec_rows[i] < M, LLX_ERR_RANGE, "record row outside the launch");
    } else {
      n_rec = M;
    }
    cudaSetDevice(s->m->device);
    stage_tokens(s, tokens, s->B * M);
    const bool identity = !rec_rows || n_rec == M;
    if (M == 1 && identity) {
      cudaGraphExec_t g = build_decode_graph(s, logits != nullptr);
      set_pos(s, pos);
      LLX_CUDA(cudaGraphLaunch(g, s->st));
      s->last_R = s->last_Rtail = s->B;
      s->last_tail = false;
      s->last_logits = logits != nullptr;
    } else {
      run_launch(s, M, pos, true, rec_rows, n_rec);
    }
    check_device_error(s);
    copy_outputs(s, s->B * n_rec, logits, argmax);
  });
}

llx_status llx_run_rows(llx_session* s, const int16_t* rows, int M, int pos, int16_t* logits, int32_t* argmax) {
  return guarded([&] {
    require(s && rows, LLX_ERR_INVALID, "null argument");
    require(M >= 1 && M <= s->max_rows, LLX_ERR_RANGE, "M outside [1, max_rows]");
    require(pos >= 0 && pos + M <= s->m->max_seq, LLX_ERR_RANGE,
            "positions " + std::to_string(pos) + ".." + std::to_string(pos + M - 1) +
                " exceed max_seq=" + std::to_string(s->m->max_seq));
    cudaSetDevice(s->m->device);
    const size_t n = (size_t)s->B * M * s->m->dim;
    LLX_CUDA(cudaStreamSynchronize(s->st));
    ensure_i16(s, n);
    std::memcpy(s->h_i16, rows, n * sizeof(int16_t));
    const Binding bd = bind(s, false);
    LLX_CUDA(cudaMemcpyAsync(bd.p[s->m->input_act], s->h_i16, n * sizeof(int16_t), cudaMemcpyHostToDevice, s->st));
    LLX_CUDA(cudaMemsetAsync(s->d_amax_key, 0, sizeof(unsigned long long) * s->B * M, s->st));
    run_launch(s, M, pos, false, nullptr, M);
    copy_outputs(s, s->B * M, logits, argmax);
  });
}

llx_status llx_generate(llx_session* s, const int32_t* prompts, int L, int n_tokens, int prefill_rows,
                        int32_t* generated, int32_t* argmax, int16_t* logits, int* n_launch_out) {
  return guarded([&] {
    require(s && prompts && generated && argmax, LLX_ERR_INVALID, "null argument");
    llx_model* m = s->m;
    require(n_tokens >= 0, LLX_ERR_INVALID, "n_tokens must be a nonnegative integer");
    require(L >= 1, LLX_ERR_INVALID, "empty prompt");
    require(L + n_tokens <= m->max_seq, LLX_ERR_RANGE,
            "prompt + tokens = " + std::to_string(L + n_tokens) + " exceeds max_seq=" + std::to_string(m->max_seq));
    const int pm = m->prefill_m;
    if (prefill_rows > 0) {
      require(prefill_rows % pm == 0, LLX_ERR_INVALID, "prefill_rows must be a multiple of prefill_m");
      require(prefill_rows <= s->max_rows, LLX_ERR_RANGE, "prefill_rows exceeds the session's max_rows");
    } else {
      require(pm <= s->max_rows, LLX_ERR_RANGE, "prefill_m exceeds the session's max_rows");
    }
    const int B = s->B;
    for (int i = 0; i < B * L; ++i)
      require(prompts[i] >= 0 && prompts[i] < m->vocab, LLX_ERR_RANGE, "prompt token ID exceeds model vocabulary");
    cudaSetDevice(m->device);
    reset_kv(s);
    const int n_chunks = (L + pm - 1) / pm;
    const int n_dec = std::min(n_tokens, std::max(0, m->max_seq - L - 1));
    const int n_launch = n_chunks + n_dec;
    *n_launch_out = n_launch;
    const int V = m->vocab, VP = m->vocab_padded_full;
    std::vector<int32_t> tok, rec, am;
    std::vector<int16_t> lg;
    // ---- prefill: golden chunks c = 0..n_chunks-1, grouped into launches ----
    const int chunks_per_launch = prefill_rows > 0 ? prefill_rows / pm : 1;
    for (int c0 = 0; c0 < n_chunks; c0 += chunks_per_launch) {
      const int c1 = std::min(n_chunks, c0 + chunks_per_launch);
      const int p0 = c0 * pm;
      const int M = prefill_rows > 0 ? std::min(L, c1 * pm) - p0 : pm;  // golden mode pads to pm rows
      const int nr = c1 - c0;
      tok.assign((size_t)B * M, -1);
      for (int b = 0; b < B; ++b)
        for (int r = 0; r < M && p0 + r < L; ++r) tok[(size_t)b * M + r] = prompts[(size_t)b * L + p0 + r];
      rec.resize((size_t)B * nr);
      for (int b = 0; b < B; ++b)
        for (int c = c0; c < c1; ++c) rec[(size_t)b * nr + (c - c0)] = std::min(L, (c + 1) * pm) - 1 - p0;
      stage_tokens(s, tok.data(), B * M);
      run_launch(s, M, p0, true, rec.data(), nr);
      check_device_error(s);
      am.resize((size_t)B * nr);
      if (logits) lg.resize((size_t)B * nr * VP);
      copy_outputs(s, B * nr, logits ? lg.data() : nullptr, am.data());
      for (int b = 0; b < B; ++b)
        for (int j = 0; j < nr; ++j) {
          argmax[(size_t)b * n_launch + c0 + j] = am[(size_t)b * nr + j];
          if (logits)
            std::memcpy(logits + ((size_t)b * n_launch + c0 + j) * V, lg.data() + ((size_t)b * nr + j) * VP,
                        sizeof(int16_t) * V);
        }
    }
    // ---- decode: first token = argmax of the last prefill chunk ----
    std::vector<int32_t> nxt(B);
    for (int b = 0; b < B; ++b) nxt[b] = argmax[(size_t)b * n_launch + n_chunks - 1];
    if (n_tokens > 0)
      for (int b = 0; b < B; ++b) generated[(size_t)b * n_tokens] = nxt[b];
    if (n_dec > 0) {
      cudaGraphExec_t g = build_decode_graph(s, logits != nullptr);
      s->last_logits = logits != nullptr;
      stage_tokens(s, nxt.data(), B);
      set_pos(s, L);
      if (logits) lg.resize((size_t)B * VP);
      for (int i = 0; i < n_dec; ++i) {
        LLX_CUDA(cudaGraphLaunch(g, s->st));
        if (logits) {
          fetch_logits(s, B, lg.data());
          for (int b = 0; b < B; ++b)
            std::memcpy(logits + ((size_t)b * n_launch + n_chunks + i) * V, lg.data() + (size_t)b * VP,
                        sizeof(int16_t) * V);
        }
      }
      std::vector<int32_t> hist((size_t)n_dec * B);
      LLX_CUDA(cudaMemcpyAsync(hist.data(), s->d_hist, sizeof(int32_t) * hist.size(), cudaMemcpyDeviceToHost, s->st));
      LLX_CUDA(cudaStreamSynchronize(s->st));
      check_device_error(s);
      for (int i = 0; i < n_dec; ++i)
        for (int b = 0; b < B; ++b) {
          const int32_t t = hist[(size_t)i * B + b];
          argmax[(size_t)b * n_launch + n_chunks + i] = t;
          if (i + 1 < n_tokens) generated[(size_t)b * n_tokens + i + 1] = t;
        }
    }
  });
}

llx_status llx_set_tokens(llx_session* s, const int32_t* tokens) {
  return guarded([&] {
    require(s && tokens, LLX_ERR_INVALID, "null argument");
    cudaSetDevice(s->m->device);
    stage_tokens(s, tokens, s->B);
  });
}

llx_status llx_decode_async(llx_session* s, int pos, int n_steps) {
  return guarded([&] {
    require(s, LLX_ERR_INVALID, "null session");
    require(n_steps >= 0 && pos >= 0 && pos + n_steps <= s->m->max_seq, LLX_ERR_RANGE,
            "decode positions exceed max_seq");
    cudaSetDevice(s->m->device);
    cudaGraphExec_t g = build_decode_graph(s, false);
    s->last_logits = false;
    set_pos(s, pos);
    for (int i = 0; i < n_steps; ++i) LLX_CUDA(cudaGraphLaunch(g, s->st));
  });
}

llx_status llx_read_history(llx_session* s, int n_steps, int32_t* history) {
  return guarded([&] {
    require(s && history, LLX_ERR_INVALID, "null argument");
    require(n_steps >= 0 && n_steps <= s->hist_cap, LLX_ERR_RANGE, "history holds max_seq steps");
    LLX_CUDA(cudaMemcpyAsync(history, s->d_hist, sizeof(int32_t) * n_steps * s->B, cudaMemcpyDeviceToHost, s->st));
    LLX_CUDA(cudaStreamSynchronize(s->st));
  });
}

llx_status llx_sync(llx_session* s) {
  return guarded([&] {
    require(s, LLX_ERR_INVALID, "null session");
    LLX_CUDA(cudaStreamSynchronize(s->st));
    check_device_error(s);
  });
}

void* llx_session_stream(llx_session* s) { return s ? (void*)s->st : nullptr; }

int llx_decode_launches_per_step(llx_session* s) {
  if (!s) return -1;
  if (!s->decode_exec[0]) {
    try {
      build_decode_graph(s, false);
    } catch (const std::exception& e) {
      g_err = e.what();
      return -1;
    }
  }
  return s->decode_launches;
}

int llx_plan_steps(const llx_model* m) { return m ? (int)m->steps.size() + 1 : 0; }

const char* llx_step_label(const llx_model* m, int i) {
  if (!m || i < 0 || i > (int)m->steps.size()) return nullptr;
  static const char* kArgmax = "argmax";
  return i == (int)m->steps.size() ? kArgmax : m->steps[i].label.c_str();
}

// the L2 flush of llx_profile_decode: twice the B200's 126 MB L2
static constexpr size_t kFlushBytes = (size_t)256 << 20;

llx_status llx_profile_decode(llx_session* s, int pos, int iters, float* ms, double* bytes, double* ops, int n_max,
                              int* n_out) {
  return guarded([&] {
    require(s && ms && bytes && ops && n_out, LLX_ERR_INVALID, "null argument");
    require(iters >= 1, LLX_ERR_INVALID, "iters must be >= 1");
    require(pos >= 0 && pos < s->m->max_seq, LLX_ERR_RANGE, "pos outside [0, max_seq)");
    llx_model* m = s->m;
    cudaSetDevice(m->device);
    set_pos(s, pos);
    const Binding bd = bind(s, false);
    const int R = s->B;
    cudaEvent_t e0, e1;
    LLX_CUDA(cudaEventCreate(&e0));
    LLX_CUDA(cudaEventCreate(&e1));
    if (!s->d_flush) LLX_CUDA(cudaMalloc(&s->d_flush, kFlushBytes));
    const int n = std::min<int>(n_max, (int)m->steps.size() + 1);
    const double T = pos + 1;
    for (int i = 0; i < n; ++i) {
      double b = 0, o = 0;
      if (i < (int)m->steps.size()) {
        const Step& x = m->steps[i];
        auto cols = [&](int a) { return (double)m->acts[a].cols; };
        switch (x.kind) {
          case SK::Embed: b = R * (4.0 + 4.0 * m->dim); break;
          case SK::RmsNorm: b = 2.0 * x.K + R * cols(x.in) * (x.out2 >= 0 ? 5.0 : 4.0); break;
          case SK::Quant: b = R * cols(x.in) * 3.0; break;
          case SK::Linear:
            // the decode loop's output linear stores no logits (argmax keys only)
            b = (double)x.N * x.K + 8.0 * x.N + (x.bias_off >= 0 ? 4.0 * x.N : 0.0) + (double)R * x.K +
                (x.out == m->output_act && output_argmax_fused(m, R) ? 0.0 : (double)R * x.N * (x.out_i8 ? 1 : 2)) +
                (x.in2 >= 0 ? 2.0 * R * x.N : 0.0);
            o = 2.0 * R * x.N * x.K;
            break;
          case SK::Rope:
            b = R * x.H * x.D * (x.out2 >= 0 ? 5.0 : 4.0) + R * 2.0 * x.D + (x.write_k ? 1.0 * R * x.H * x.D : 0.0);
            break;
          case SK::KvWrite: b = (x.in >= 0 ? 2.0 : 1.0) * 2.0 * R * x.Hkv * x.D; break;
          case SK::LinearPartial:
            b = (double)x.N * x.K + (double)R * x.K + 4.0 * R * x.N;
            o = 2.0 * R * x.N * x.K;
            break;
          case SK::AllReduce: b = 8.0 * R * x.N; break;  // read + write of the local buffer
          case SK::Requant:
            b = 4.0 * R * x.N + 8.0 * x.N + (x.bias_off >= 0 ? 4.0 * x.N : 0.0) + (double)R * x.N * (x.out_i8 ? 1 : 2) +
                (x.in2 >= 0 ? 2.0 * R * x.N : 0.0);
            break;
          case SK::Attention:
            b = 2.0 * R * x.Hkv * T * x.D + 2.0 * R * x.H * x.D;
            o = 4.0 * R * x.H * x.D * T;
            break;
          case SK::Add:
          case SK::Mul: b = 6.0 * R * cols(x.in); break;
          case SK::Silu: b = 4.0 * R * cols(x.in); break;
          case SK::LinearGroup:
          case SK::Gated:
            for (const Step& p : x.parts) {
              if (p.kind == SK::Linear) {
                b += (double)p.N * p.K + 8.0 * p.N + (p.bias_off >= 0 ? 4.0 * p.N : 0.0) +
                     (double)R * p.N * (p.out_i8 ? 1 : 2);
                o += 2.0 * R * p.N * p.K;
              } else if (p.kind == SK::Quant) {
                b += (double)R * cols(p.out);
              }
            }
            if (x.kind == SK::Gated) b -= 2.0 * R * x.parts[0].N;  // the gate output is not re-read
            b += (double)R * x.K;
            break;
          case SK::RopeGroup:
            for (const Step& p : x.parts) {
              if (p.kind == SK::Rope)
                b += R * p.H * p.D * 5.0 + R * 2.0 * p.D + (p.write_k ? 1.0 * R * p.H * p.D : 0.0);
              else
                b += 2.0 * R * p.Hkv * p.D;
            }
            break;
        }
      } else {
        b = output_argmax_fused(m, R) ? 12.0 * R : 2.0 * R * m->vocab_padded + 4.0 * R;
      }
      // one untimed launch, then `iters` timed launches, each alone between two events after
      // a write of twice the L2 size (its inputs come from HBM, as in the decode chain); a
      // step folded into a neighbour (it launches nothing at M = 1) reports zero time and bytes
      int launched = 1;
      float total = 0.0f;
      s->store_logits = false;  // as in the decode loop's graph
      try {
        for (int it = 0; it <= iters; ++it) {
          LLX_CUDA(cudaMemsetAsync(s->d_flush, it & 1, kFlushBytes, s->st));
          LLX_CUDA(cudaEventRecord(e0, s->st));
          if (i < (int)m->steps.size()) {
            launched = enqueue_steps(s, bd, i, i + 1, R, 1);
          } else {
            launch_output_argmax(s, bd.p[m->output_act], R);
          }
          LLX_CUDA(cudaEventRecord(e1, s->st));
          LLX_CUDA(cudaEventSynchronize(e1));
          float t = 0;
          LLX_CUDA(cudaEventElapsedTime(&t, e0, e1));
          if (it > 0) total += t;
        }
      } catch (...) {
        s->store_logits = true;
        throw;
      }
      s->store_logits = true;
      s->last_logits = false;
      if (launched == 0) b = o = 0;
      ms[i] = launched ? total / iters : 0.0f;
      bytes[i] = b;
      ops[i] = o;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *n_out = n;
  });
}

int llx_activation_count(const llx_model* m) { return m ? (int)m->acts.size() : 0; }
const char* llx_activation_name(const llx_model* m, int i) {
  if (!m || i < 0 || i >= (int)m->acts.size()) return nullptr;
  return m->acts[i].name.c_str();
}

llx_status llx_activation_shape(const llx_model* m, const char* name, int* cols, int* elem) {
  return guarded([&] {
    require(m && name, LLX_ERR_INVALID, "null argument");
    auto it = m->act_id.find(name);
    require(it != m->act_id.end(), LLX_ERR_INVALID, std::string("unknown activation ") + name);
    if (cols) *cols = m->acts[it->second].cols;
    if (elem) *elem = m->acts[it->second].elem;
  });
}

llx_status llx_read_activation(llx_session* s, const char* name, void* dst, size_t bytes, int* rows_out) {
  return guarded([&] {
    require(s && name && dst, LLX_ERR_INVALID, "null argument");
    llx_model* m = s->m;
    auto it = m->act_id.find(name);
    require(it != m->act_id.end(), LLX_ERR_INVALID, std::string("unknown activation ") + name);
    const int a = it->second;
    require(s->keep || a == m->output_act, LLX_ERR_INVALID, "activation buffers are reused; create the session with keep_acts=1");
    require(a != m->output_act || s->last_logits, LLX_ERR_INVALID,
            "the last launch recorded only the argmax (no logits were stored)");
    bool in_tail = false;
    for (size_t i = m->tail_start; i < m->steps.size(); ++i)
      for (int o : step_outs(m->steps[i]))
        if (o == a) in_tail = true;
    const int rows = (s->last_tail && in_tail) ? s->last_Rtail : s->last_R;
    const size_t need = (size_t)rows * m->acts[a].cols * m->acts[a].elem;
    require(bytes >= need, LLX_ERR_INVALID, "destination too small");
    LLX_CUDA(cudaStreamSynchronize(s->st));
    LLX_CUDA(cudaMemcpy(dst, s->arena + s->act_off[a], need, cudaMemcpyDeviceToHost));
    if (rows_out) *rows_out = rows;
  });
}

}  // extern "C"
