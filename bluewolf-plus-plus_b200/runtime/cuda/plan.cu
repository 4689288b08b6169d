// Launch-plan executor: runs a graph built by the reference compiler on the
// B200 kernels, either from the launch plan that `bwppc --target cuda`
// writes (compiler/codegen_cuda.c of this package: fusion decisions, operand
// value ids and arena offsets all made by the compiler; parse_launch below),
// or from the compiler's own dumps, lowered here:
//   bwppc <in.bwpp> <out.metal> --entry <fn> --dot g.dot [--mem-plan m.txt]
//   bwppc ... --grad-dot g.dot                     (the gradient graph)
// The graph dump (compiler/graph_ir.c:1326-1358) lists every value (name,
// dtype, symbolic shape, input / output flag) and every node (op, input
// edges in order, output); the memory-plan dump (compiler/mem_plan.c:176-193)
// maps values to shared buffers (greedy reuse, compiler/mem_plan.c:43-146).
// Symbolic dims are bound at plan creation ("T=128,D=256,...").
//
// Lowering (at creation, once):
//   * matmul(q, transpose(k)) -> softmax -> matmul(., v) becomes one call of
//     the attention kernel (no [T, T] scores in memory; unscaled, unmasked as
//     the graph states, compiler/graph_ir.c:1852-1899 pattern);
//   * a transpose feeding only matmuls is folded into the GEMM operand layout
//     (K-major B / MN-major A): no transposed copy;
//   * matmul -> add(., [N] or reshape of [N]) -> silu -> add(., R) fuses into
//     the GEMM epilogue (bias, SiLU, residual): bias found by dataflow, so the
//     reshape(bias) form the reference's fusion pass misses
//     (compiler/graph_ir.c:760-767, compiler/codegen_metal.c:17-123) fuses
//     too;
//   * mul(silu(x), y) becomes one swiglu pass and rmsnorm(add(a, b)) one
//     residual + norm row pass;
//   * everything else is one kernel per node (plan_ops.cu, half_ops.cu,
//     norms.cu, reduce_max.cu), permute and the reduce_max family included
//     (from dumps, a permute's axes are read off the symbolic dims).
// A fusion is skipped when the memory plan hands one of its inputs' buffers
// to a value produced before the fused step runs.  A GEMM / attention /
// transpose / reduction whose output the plan puts in one of its inputs'
// buffers gets a buffer of its own instead (they do not run in place).  Values keep the graph's dtype (f16, bf16 or f32);
// arithmetic is fp32; GEMM and attention take f16 operands as f16 and f32
// operands rounded to bf16.
#include <ctype.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "bwpp_cuda_internal.cuh"

int bwpp_gemm_launch_dt(BwppCudaCtx *ctx, const uint16_t *a, int a_mn, uint32_t lda,
                        const uint16_t *b, int b_mn, uint32_t ldb, void *c, uint32_t ldc,
                        uint32_t M, uint32_t N, uint32_t K, const float *bias, int silu,
                        const void *residual, uint32_t ldr, int out_bf16, int force_simt,
                        int ab_f16, int out_f16, int res16);
int bwpp_attention_launch(BwppCudaCtx *ctx, const uint16_t *q, const uint16_t *k,
                          const uint16_t *v, void *o, uint32_t BH, uint32_t Sq, uint32_t Skv,
                          uint32_t Kd, uint32_t Dv, uint64_t q_bh, uint64_t k_bh, uint64_t v_bh,
                          uint64_t o_bh, uint32_t ldq, uint32_t ldk, uint32_t ldv, uint32_t ldo,
                          float scale, int causal, int f16);
int bwpp_plan_binary(BwppCudaCtx *ctx, int dt, const void *a, const void *b, void *o, uint32_t R,
                     uint32_t C, int op, int bmode);
int bwpp_plan_unary(BwppCudaCtx *ctx, int dt, const void *x, void *o, size_t n, int op);
int bwpp_plan_convert(BwppCudaCtx *ctx, int di, int dout, const void *x, void *o, size_t n);
int bwpp_plan_silu_grad(BwppCudaCtx *ctx, int dt, const void *x, const void *dy, void *dx,
                        size_t n);
int bwpp_plan_softmax_grad(BwppCudaCtx *ctx, int dt, const void *y, const void *dy, void *dx,
                           uint32_t R, uint32_t C);
int bwpp_plan_rmsnorm_grad(BwppCudaCtx *ctx, int dt, const void *x, const void *gamma,
                           const void *dy, void *dx, uint32_t R, uint32_t C, float eps);
int bwpp_plan_softmax(BwppCudaCtx *ctx, int dt, const void *x, void *y, uint32_t R, uint32_t C);
int bwpp_plan_rmsnorm(BwppCudaCtx *ctx, int dt, const void *x, const void *gamma,
                      const void *beta, void *y, uint32_t R, uint32_t C, float eps);
int bwpp_plan_reduce_sum(BwppCudaCtx *ctx, int dt, const void *x, void *o, uint32_t R, uint32_t C,
                         int axis);
int bwpp_plan_transpose(BwppCudaCtx *ctx, int dt, const void *x, void *o, uint32_t batch,
                        uint32_t R, uint32_t C);
int bwpp_plan_swiglu(BwppCudaCtx *ctx, int dt, const void *a, const void *b, void *o, size_t n);
int bwpp_plan_permute(BwppCudaCtx *ctx, int dt, const void *x, void *o, int rank,
                      const int64_t *dims, const int *perm);
int bwpp_plan_reduce_max(BwppCudaCtx *ctx, int dt, const void *x, void *o, uint32_t outer,
                         uint32_t n, uint32_t inner, int mode);
int bwpp_plan_add_rmsnorm(BwppCudaCtx *ctx, int dt, const void *a, const void *b,
                          const void *gamma, const void *beta, void *h, void *y, uint32_t R,
                          uint32_t C, float eps);

namespace {

enum { DT_F16 = 0, DT_BF16 = 1, DT_F32 = 2 };
size_t dt_size(int dt) { return dt == DT_F32 ? 4 : 2; }
const char *dt_name(int dt) { return dt == DT_F16 ? "f16" : dt == DT_BF16 ? "bf16" : "f32"; }

thread_local char tl_err[512];

struct Val {
  int id = -1;
  std::string name;
  int dtype = DT_F16;
  std::vector<std::string> sdims;
  std::vector<int64_t> dims;
  bool known = false;
  bool input = false, output = false;
  int producer = -1;            // node position
  std::vector<int> uses;        // node positions, one per input edge
  int buffer = -1;              // memory-plan buffer, -1: none
  bool live = true;             // false: fused away, never materialised
  void *ptr = nullptr;
  bool bound = false;
  size_t off = SIZE_MAX;        // arena offset given by a launch plan
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : dims) n *= d;
    return n;
  }
  int64_t last() const { return dims.empty() ? 1 : dims.back(); }
  int64_t rows() const { return dims.empty() ? 1 : numel() / std::max<int64_t>(1, last()); }
};

struct Node {
  int id = -1;
  std::string op;
  std::vector<int> in;
  int out = -1;
  bool fused = false;  // consumed by a fused step
};

enum Kind {
  K_GEMM, K_ATTN, K_SOFTMAX, K_RMSNORM, K_UNARY, K_BINARY, K_TRANSPOSE, K_SILU_GRAD,
  K_SOFTMAX_GRAD, K_RMSNORM_GRAD, K_REDUCE, K_SWIGLU, K_ADD_RMSNORM, K_PERMUTE, K_REDUCE_MAX
};

struct Step {
  Kind kind;
  int pos = -1;                         // node position it runs at
  int a = -1, b = -1, c = -1, out = -1; // value ids
  int a_t = 0, b_t = 0, bias = -1, silu = 0;  // GEMM: operand read transposed
  int res_mul = 0;                      // GEMM: c multiplies (SwiGLU gate) instead of adding
  int d = -1, e = -1, out2 = -1;        // add+rmsnorm: gamma, beta, the stored sum (or -1)
  float eps = 1e-5f;                    // rmsnorm, rmsnorm_grad, add+rmsnorm
  int perm[4] = {0, 1, 2, 3};           // permute: input dim of each output dim
  int op = 0, bmode = 0, axis = 1;
  size_t bias_off = 0;                  // fp32 bias scratch offset
  std::string what;
};

bool starts_with(const char *s, const char *p) { return strncmp(s, p, strlen(p)) == 0; }

std::string trim(const std::string &s) {
  size_t a = 0, b = s.size();
  while (a < b && isspace((unsigned char)s[a])) ++a;
  while (b > a && isspace((unsigned char)s[b - 1])) --b;
  return s.substr(a, b - a);
}

int parse_dtype(const std::string &s) {
  if (s == "f16") return DT_F16;
  if (s == "bf16") return DT_BF16;
  if (s == "f32") return DT_F32;
  return -1;
}

std::vector<std::string> split_dims(const std::string &inner) {
  std::vector<std::string> out;
  std::string cur;
  for (char ch : inner) {
    if (ch == ',') {
      out.push_back(trim(cur));
      cur.clear();
    } else {
      cur += ch;
    }
  }
  if (!trim(cur).empty()) out.push_back(trim(cur));
  return out;
}

}  // namespace

struct BwppCudaPlan {
  BwppCudaCtx *ctx = nullptr;
  std::vector<Val> vals;
  std::vector<Node> nodes;
  std::vector<Step> steps;
  std::map<std::string, int64_t> dims;
  std::vector<int> mp_buf;              // value id -> memory-plan buffer
  int mp_buffers = 0;
  float eps = 1e-5f;
  int fuse = 1;
  bool from_launch = false;             // built from a `bwppc --target cuda` plan
  size_t graph_bytes = 0;               // its arena bytes (graph values)
  // device memory: one allocation
  uint8_t *arena = nullptr;
  size_t arena_bytes = 0;
  size_t scratch_off = 0, scratch_bytes = 0;  // aliased outputs / casts
  size_t launches = 0;
  std::string err;

  int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    err = buf;
    snprintf(tl_err, sizeof(tl_err), "%s", buf);
    if (ctx) bwpp_set_error(ctx, code, "plan: %s", buf);
    return code;
  }

  Val *val(int id) { return (id >= 0 && id < (int)vals.size() && vals[id].id >= 0) ? &vals[id] : nullptr; }

  // ---------------------------------------------------------------- parsing
  int parse_graph(const char *text) {
    const char *p = text;
    std::map<int, int> node_pos;  // node id -> position
    while (*p) {
      const char *eol = strchr(p, '\n');
      std::string line = trim(std::string(p, eol ? eol - p : strlen(p)));
      p = eol ? eol + 1 : p + strlen(p);
      if (line.empty()) continue;
      int a = -1, b = -1;
      if (line[0] == 'v' && isdigit((unsigned char)line[1]) &&
          line.find("[shape=ellipse") != std::string::npos) {
        Val v;
        v.id = atoi(line.c_str() + 1);
        v.input = line.find("#E7F0FF") != std::string::npos;
        v.output = line.find("#E8FFE7") != std::string::npos;
        const size_t l0 = line.find("label=\"");
        const size_t l1 = line.rfind("\"]");
        if (l0 == std::string::npos || l1 == std::string::npos || l1 < l0 + 7)
          return fail(BWPP_CUDA_ERR_ARG, "bad value line: %s", line.c_str());
        std::string label = line.substr(l0 + 7, l1 - (l0 + 7));
        const size_t nl = label.find("\\n");
        if (nl != std::string::npos) {
          v.name = label.substr(0, nl);
          label = label.substr(nl + 2);
        }
        const size_t sp = label.find(' ');
        const size_t lb = label.find('['), rb = label.rfind(']');
        if (sp == std::string::npos || lb == std::string::npos || rb == std::string::npos)
          return fail(BWPP_CUDA_ERR_ARG, "bad value label: %s", label.c_str());
        v.dtype = parse_dtype(label.substr(0, sp));
        if (v.dtype < 0) return fail(BWPP_CUDA_ERR_UNSUPPORTED, "dtype %s", label.substr(0, sp).c_str());
        v.sdims = split_dims(label.substr(lb + 1, rb - lb - 1));
        if (v.id >= (int)vals.size()) vals.resize(v.id + 1);
        vals[v.id] = v;
      } else if (line[0] == 'n' && isdigit((unsigned char)line[1]) &&
                 line.find("[shape=box") != std::string::npos) {
        Node n;
        n.id = atoi(line.c_str() + 1);
        const size_t l0 = line.find("label=\"");
        const size_t l1 = line.rfind("\"]");
        if (l0 == std::string::npos || l1 == std::string::npos)
          return fail(BWPP_CUDA_ERR_ARG, "bad node line: %s", line.c_str());
        n.op = line.substr(l0 + 7, l1 - (l0 + 7));
        node_pos[n.id] = (int)nodes.size();
        nodes.push_back(n);
      } else if (sscanf(line.c_str(), "v%d -> n%d;", &a, &b) == 2 && line[0] == 'v') {
        auto it = node_pos.find(b);
        if (it == node_pos.end()) return fail(BWPP_CUDA_ERR_ARG, "edge to unknown node n%d", b);
        nodes[it->second].in.push_back(a);
      } else if (sscanf(line.c_str(), "n%d -> v%d;", &a, &b) == 2 && line[0] == 'n') {
        auto it = node_pos.find(a);
        if (it == node_pos.end()) return fail(BWPP_CUDA_ERR_ARG, "edge from unknown node n%d", a);
        nodes[it->second].out = b;
      }
    }
    if (nodes.empty() && vals.empty()) return fail(BWPP_CUDA_ERR_ARG, "no graph in the dump");
    for (size_t i = 0; i < nodes.size(); ++i) {
      Node &n = nodes[i];
      if (!val(n.out)) return fail(BWPP_CUDA_ERR_ARG, "node n%d has no output value", n.id);
      if (vals[n.out].producer >= 0) return fail(BWPP_CUDA_ERR_ARG, "v%d produced twice", n.out);
      vals[n.out].producer = (int)i;
      for (int x : n.in) {
        if (!val(x)) return fail(BWPP_CUDA_ERR_ARG, "node n%d reads unknown v%d", n.id, x);
        vals[x].uses.push_back((int)i);
      }
    }
    for (size_t i = 0; i < nodes.size(); ++i)
      for (int x : nodes[i].in)
        if (!vals[x].input && vals[x].producer >= (int)i)
          return fail(BWPP_CUDA_ERR_ARG, "nodes are not in dependency order at n%d", nodes[i].id);
    return BWPP_CUDA_OK;
  }

  // ---------------------------------------------------- `--target cuda` plan
  // The lines of compiler/codegen_cuda.c: bwpp.value (id, name, dtype, bound
  // dims, flags, buffer, arena offset), bwpp.arena (bytes) and bwpp.launch
  // (kernel, operands, epilogue), in launch order.  Nothing is re-lowered.
  static std::map<std::string, std::string> kv_fields(const std::string &line, size_t from) {
    std::map<std::string, std::string> kv;
    size_t i = from;
    while (i < line.size()) {
      while (i < line.size() && isspace((unsigned char)line[i])) ++i;
      size_t j = i;
      while (j < line.size() && !isspace((unsigned char)line[j])) ++j;
      const std::string tok = line.substr(i, j - i);
      const size_t eq = tok.find('=');
      if (eq != std::string::npos) kv[tok.substr(0, eq)] = tok.substr(eq + 1);
      i = j;
    }
    return kv;
  }

  static int vref(const std::string &t) {  // "v12" -> 12, else -1
    if (t.size() < 2 || t[0] != 'v' || !isdigit((unsigned char)t[1])) return -1;
    return atoi(t.c_str() + 1);
  }

  int parse_launch(const char *text) {
    from_launch = true;
    bool have_arena = false;
    std::vector<std::string> launches;
    const char *p = text;
    while (*p) {
      const char *eol = strchr(p, '\n');
      std::string line = trim(std::string(p, eol ? eol - p : strlen(p)));
      p = eol ? eol + 1 : p + strlen(p);
      if (starts_with(line.c_str(), "// bwpp.value: ")) {
        const size_t at = strlen("// bwpp.value: ");
        const size_t sp = line.find(' ', at);
        Val v;
        v.id = vref(line.substr(at, sp == std::string::npos ? std::string::npos : sp - at));
        if (v.id < 0 || v.id > (1 << 20)) return fail(BWPP_CUDA_ERR_ARG, "launch plan: bad value line %s", line.c_str());
        auto kv = kv_fields(line, sp == std::string::npos ? line.size() : sp);
        v.name = kv["name"];
        v.dtype = parse_dtype(kv["dtype"]);
        if (v.dtype < 0) return fail(BWPP_CUDA_ERR_UNSUPPORTED, "launch plan: v%d dtype", v.id);
        for (const auto &d : split_dims(kv["dims"])) {
          const long long n = atoll(d.c_str());
          if (n <= 0) return fail(BWPP_CUDA_ERR_ARG, "launch plan: v%d dims", v.id);
          v.dims.push_back(n);
        }
        v.known = !v.dims.empty();
        const std::string &fl = kv["flags"];
        v.input = fl.find("input") != std::string::npos;
        v.output = fl.find("output") != std::string::npos;
        v.live = v.input || kv.count("offset");
        if (kv.count("buffer") && kv["buffer"][0] == 'b') {
          v.buffer = atoi(kv["buffer"].c_str() + 1);
          mp_buffers = std::max(mp_buffers, v.buffer + 1);
        }
        if (kv.count("offset")) v.off = (size_t)strtoull(kv["offset"].c_str(), nullptr, 10);
        if (v.id >= (int)vals.size()) vals.resize(v.id + 1);
        vals[v.id] = v;
      } else if (starts_with(line.c_str(), "// bwpp.arena: bytes=")) {
        graph_bytes = (size_t)strtoull(line.c_str() + strlen("// bwpp.arena: bytes="), nullptr, 10);
        have_arena = true;
      } else if (starts_with(line.c_str(), "// bwpp.launch: ")) {
        launches.push_back(line);
      }
    }
    if (vals.empty() || !have_arena)
      return fail(BWPP_CUDA_ERR_ARG, "not a launch plan (no bwpp.value / bwpp.arena lines)");
    for (const std::string &line : launches) {
      const size_t at = strlen("// bwpp.launch: ");
      char kind[32] = {0};
      int idx = -1;
      if (sscanf(line.c_str() + at, "%d %31s", &idx, kind) != 2)
        return fail(BWPP_CUDA_ERR_ARG, "launch plan: bad launch line %s", line.c_str());
      auto kv = kv_fields(line, at);
      auto V = [&](const char *key) { return kv.count(key) ? vref(kv[key]) : -1; };
      Step st;
      const std::string k = kind;
      st.out = V("out");
      st.pos = kv.count("node") ? atoi(kv["node"].c_str() + 1) : idx;
      if (kv.count("eps")) st.eps = (float)atof(kv["eps"].c_str());
      if (k == "gemm") {
        st.kind = K_GEMM;
        st.a = V("a");
        st.b = V("b");
        st.a_t = kv.count("a_t") ? atoi(kv["a_t"].c_str()) : 0;
        st.b_t = kv.count("b_t") ? atoi(kv["b_t"].c_str()) : 0;
        st.bias = V("bias");
        st.silu = kv.count("silu") ? atoi(kv["silu"].c_str()) : 0;
        st.c = kv.count("gate") ? V("gate") : V("residual");
        st.res_mul = kv.count("gate") ? 1 : 0;
        st.what = "gemm";
        if (st.a_t) st.what += " A^T";
        if (st.b_t) st.what += " B^T";
        if (st.bias >= 0) st.what += " +bias";
        if (st.silu) st.what += " +silu";
        if (st.c >= 0) st.what += st.res_mul ? " +swiglu" : " +residual";
      } else if (k == "attention") {
        st.kind = K_ATTN;
        st.a = V("q");
        st.b = V("k");
        st.c = V("v");
        if ((kv.count("scale") && atof(kv["scale"].c_str()) != 1.0) ||
            (kv.count("causal") && atoi(kv["causal"].c_str()) != 0))
          return fail(BWPP_CUDA_ERR_UNSUPPORTED, "launch plan: scaled / causal graph attention");
        st.what = "attention (fused transpose, matmul, softmax, matmul)";
      } else if (k == "softmax") {
        st.kind = K_SOFTMAX; st.a = V("x"); st.what = "softmax";
      } else if (k == "rmsnorm") {
        st.kind = K_RMSNORM; st.a = V("x"); st.b = V("gamma"); st.c = V("beta"); st.what = "rmsnorm";
      } else if (k == "add_rmsnorm") {
        st.kind = K_ADD_RMSNORM;
        st.a = V("a"); st.b = V("b"); st.d = V("gamma"); st.e = V("beta"); st.out2 = V("sum");
        st.what = st.out2 >= 0 ? "add+rmsnorm (fused residual add and norm, sum stored)"
                               : "add+rmsnorm (fused residual add and norm)";
      } else if (k == "swiglu") {
        st.kind = K_SWIGLU; st.a = V("x"); st.b = V("y"); st.what = "swiglu (fused silu, mul)";
      } else if (k == "unary") {
        st.kind = K_UNARY;
        st.a = V("x");
        st.op = kv["op"] == "silu" ? 1 : 0;
        st.what = st.op ? "silu" : "reshape";
      } else if (k == "binary") {
        static const char *ops[] = {"add", "sub", "mul", "div", "broadcast"};
        st.kind = K_BINARY;
        st.a = V("a");
        st.b = V("b");
        st.op = -1;
        for (int o = 0; o < 5; ++o)
          if (kv["op"] == ops[o]) st.op = o;
        if (st.op < 0) return fail(BWPP_CUDA_ERR_ARG, "launch plan: binary op %s", kv["op"].c_str());
        st.what = ops[st.op];
      } else if (k == "transpose") {
        st.kind = K_TRANSPOSE; st.a = V("x"); st.what = "transpose";
      } else if (k == "silu_grad") {
        st.kind = K_SILU_GRAD; st.a = V("x"); st.b = V("dy"); st.what = "silu_grad";
      } else if (k == "softmax_grad") {
        st.kind = K_SOFTMAX_GRAD; st.a = V("y"); st.b = V("dy"); st.what = "softmax_grad";
      } else if (k == "rmsnorm_grad") {
        st.kind = K_RMSNORM_GRAD; st.a = V("x"); st.b = V("gamma"); st.c = V("dy");
        st.what = "rmsnorm_grad";
      } else if (k == "reduce_sum") {
        st.kind = K_REDUCE; st.a = V("x"); st.what = "reduce_sum";
      } else if (k == "permute") {
        st.kind = K_PERMUTE;
        st.a = V("x");
        st.what = "permute";
        const auto p = split_dims(kv["perm"]);
        if (p.empty() || p.size() > 4) return fail(BWPP_CUDA_ERR_ARG, "launch plan: permute perm");
        for (size_t i = 0; i < p.size(); ++i) st.perm[i] = atoi(p[i].c_str());
      } else if (k == "reduce_max") {
        st.kind = K_REDUCE_MAX;
        st.a = V("x");
        st.axis = kv.count("axis") ? atoi(kv["axis"].c_str()) : -1;
        st.op = kv["mode"] == "mask" ? 1 : 0;
        st.what = st.op ? "reduce_max_mask" : "reduce_max";
      } else if (k == "reduce_max_grad") {
        st.kind = K_BINARY; st.a = V("mask"); st.b = V("dy"); st.op = 2; st.what = "reduce_max_grad";
      } else {
        return fail(BWPP_CUDA_ERR_UNSUPPORTED, "launch plan: unknown kernel %s", kind);
      }
      // every operand names a known value with a bound shape
      const int need[] = {st.out, st.a};
      for (int x : need)
        if (!val(x) || !vals[x].known) return fail(BWPP_CUDA_ERR_ARG, "launch plan: %s", line.c_str());
      for (int x : {st.b, st.c, st.bias, st.d, st.e, st.out2})
        if (x != -1 && (!val(x) || !vals[x].known))
          return fail(BWPP_CUDA_ERR_ARG, "launch plan: %s", line.c_str());
      if (st.pos < 0 || st.pos > (1 << 20)) return fail(BWPP_CUDA_ERR_ARG, "launch plan: node");
      if ((int)nodes.size() <= st.pos) nodes.resize(st.pos + 1);
      for (int x : {st.a, st.b, st.c, st.bias, st.d, st.e})
        if (x >= 0) vals[x].uses.push_back(st.pos);
      steps.push_back(st);
    }
    for (size_t i = 0; i < nodes.size(); ++i) nodes[i].id = (int)i;
    return BWPP_CUDA_OK;
  }

  int parse_mem_plan(const char *text) {
    mp_buf.assign(vals.size(), -1);
    const char *p = text;
    while (*p) {
      const char *eol = strchr(p, '\n');
      std::string line = trim(std::string(p, eol ? eol - p : strlen(p)));
      p = eol ? eol + 1 : p + strlen(p);
      unsigned a = 0, b = 0;
      if (sscanf(line.c_str(), "buffers=%u values=%u", &a, &b) == 2) {
        mp_buffers = (int)a;
      } else if (line[0] == 'v' && sscanf(line.c_str(), "v%u -> buffer%u", &a, &b) == 2) {
        if ((int)a >= (int)vals.size() || (int)b >= mp_buffers)
          return fail(BWPP_CUDA_ERR_ARG, "memory plan: bad line %s", line.c_str());
        mp_buf[a] = (int)b;
      }
    }
    for (auto &v : vals)
      if (v.id >= 0 && !v.input) v.buffer = mp_buf[v.id];
    return BWPP_CUDA_OK;
  }

  int parse_dims(const char *spec) {
    if (!spec) return BWPP_CUDA_OK;
    std::string s(spec);
    size_t i = 0;
    while (i < s.size()) {
      size_t j = s.find(',', i);
      if (j == std::string::npos) j = s.size();
      std::string kv = trim(s.substr(i, j - i));
      i = j + 1;
      if (kv.empty()) continue;
      const size_t eq = kv.find('=');
      if (eq == std::string::npos) return fail(BWPP_CUDA_ERR_ARG, "dims: '%s' is not NAME=VALUE", kv.c_str());
      const long long n = atoll(kv.c_str() + eq + 1);
      if (n <= 0) return fail(BWPP_CUDA_ERR_ARG, "dims: %s must be positive", kv.c_str());
      dims[trim(kv.substr(0, eq))] = n;
    }
    return BWPP_CUDA_OK;
  }

  int parse_options(const char *spec) {
    if (!spec) return BWPP_CUDA_OK;
    std::string s(spec);
    size_t i = 0;
    while (i < s.size()) {
      size_t j = s.find(',', i);
      if (j == std::string::npos) j = s.size();
      std::string kv = trim(s.substr(i, j - i));
      i = j + 1;
      if (kv.empty()) continue;
      if (starts_with(kv.c_str(), "eps=")) eps = (float)atof(kv.c_str() + 4);
      else if (starts_with(kv.c_str(), "fuse=")) fuse = atoi(kv.c_str() + 5);
      else return fail(BWPP_CUDA_ERR_ARG, "unknown option %s", kv.c_str());
    }
    return BWPP_CUDA_OK;
  }

  // ------------------------------------------------------------------ shapes
  int resolve(Val &v) {
    if (v.sdims.empty()) return BWPP_CUDA_OK;  // rank unknown ("[]"): inferred
    v.dims.clear();
    for (const auto &d : v.sdims) {
      if (!d.empty() && isdigit((unsigned char)d[0])) {
        v.dims.push_back(atoll(d.c_str()));
      } else {
        auto it = dims.find(d);
        if (it == dims.end()) return fail(BWPP_CUDA_ERR_ARG, "dim %s of v%d is not bound", d.c_str(), v.id);
        v.dims.push_back(it->second);
      }
    }
    v.known = true;
    return BWPP_CUDA_OK;
  }

  int infer(Node &n) {
    Val &o = vals[n.out];
    std::vector<int64_t> d;
    auto in = [&](int i) -> Val & { return vals[n.in[i]]; };
    for (int x : n.in)
      if (!vals[x].known) return fail(BWPP_CUDA_ERR_ARG, "shape of v%d unknown at n%d", x, n.id);
    const std::string &op = n.op;
    if (op == "matmul" || op == "batch_matmul") {
      if (n.in.size() != 2 || in(0).dims.size() < 2 || in(1).dims.size() < 2)
        return fail(BWPP_CUDA_ERR_ARG, "n%d: matmul needs two operands of rank >= 2", n.id);
      const auto &A = in(0).dims, &B = in(1).dims;
      if (A[A.size() - 1] != B[B.size() - 2])
        return fail(BWPP_CUDA_ERR_ARG, "n%d: matmul inner dims %lld vs %lld", n.id,
                    (long long)A.back(), (long long)B[B.size() - 2]);
      d = A.size() >= B.size() ? A : B;
      d[d.size() - 2] = A[A.size() - 2];
      d[d.size() - 1] = B.back();
    } else if (op == "transpose") {
      if (in(0).dims.size() < 2) return fail(BWPP_CUDA_ERR_ARG, "n%d: transpose of rank < 2", n.id);
      d = in(0).dims;
      std::swap(d[d.size() - 1], d[d.size() - 2]);
    } else if (op == "softmax" || op == "silu" || op == "rmsnorm" || op == "silu_grad" ||
               op == "softmax_grad" || op == "rmsnorm_grad" || op == "reduce_max_mask" ||
               op == "reduce_max_grad") {
      d = in(0).dims;
    } else if (op == "add" || op == "sub" || op == "mul" || op == "div") {
      d = in(0).numel() >= in(1).numel() ? in(0).dims : in(1).dims;
    } else if (op == "reduce_sum") {
      if (o.known) return BWPP_CUDA_OK;  // the axis follows from the output shape
      d = in(0).dims;
      if (!d.empty()) d.back() = 1;
    } else {
      if (!o.known) return fail(BWPP_CUDA_ERR_UNSUPPORTED, "n%d: cannot infer the shape of %s", n.id, op.c_str());
      return BWPP_CUDA_OK;
    }
    if (o.known) {
      int64_t a = 1, b = 1;
      for (auto x : d) a *= x;
      b = o.numel();
      if (a != b)
        return fail(BWPP_CUDA_ERR_ARG, "n%d (%s): output v%d has %lld elements, inferred %lld", n.id,
                    op.c_str(), n.out, (long long)b, (long long)a);
      // the dump records some outputs untransposed (rank-4 transpose): the
      // shape that follows from the operation wins
      if (op == "transpose" || op == "matmul" || op == "batch_matmul") o.dims = d;
      return BWPP_CUDA_OK;
    }
    o.dims = d;
    o.known = true;
    return BWPP_CUDA_OK;
  }

  // -------------------------------------------------------------- lowering
  // Only use of v is by node position `pos` (once), and v is no graph output.
  bool sole_use(int v, int pos) const {
    const Val &x = vals[v];
    return !x.output && x.uses.size() == 1 && x.uses[0] == pos;
  }

  // True when running a step at `at` that reads `inputs` (instead of their
  // original readers from `from` on) is safe under the memory plan: no node
  // in [from, at) outside `group` writes a buffer one of the inputs lives in.
  bool safe_to_defer(const std::vector<int> &inputs, int from, int at,
                     const std::vector<int> &group) const {
    for (int x : inputs) {
      if (x < 0) continue;
      const Val &v = vals[x];
      if (v.input || v.buffer < 0) continue;
      for (int j = from; j < at; ++j) {
        if (std::find(group.begin(), group.end(), j) != group.end()) continue;
        if (j == v.producer) continue;
        const Val &w = vals[nodes[j].out];
        if (w.buffer == v.buffer && w.id != v.id) return false;
      }
    }
    return true;
  }

  // The rank-1 bias behind an add operand: a value of N elements, either
  // directly or through reshapes that only feed this add.
  int bias_source(int v, int64_t N, int add_pos) const {
    const Val &b = vals[v];
    if (b.numel() != N || (b.dims.size() > 2) || (b.dims.size() == 2 && b.dims[0] != 1)) return -1;
    int src = v;
    while (vals[src].producer >= 0 && nodes[vals[src].producer].op == "reshape" &&
           sole_use(src, src == v ? add_pos : -2)) {
      src = nodes[vals[src].producer].in[0];
      if (vals[src].numel() != N) return -1;
    }
    return src;
  }

  int lower() {
    const int n_nodes = (int)nodes.size();
    std::vector<int> step_at(n_nodes, -1);
    // 1. attention: transpose(k) -> matmul(q, .) -> softmax -> matmul(., v)
    if (fuse) {
      for (int pp = 0; pp < n_nodes; ++pp) {
        Node &P = nodes[pp];
        if (P.op != "softmax" || P.fused || P.in.size() != 1) continue;
        const int s = P.in[0], p = P.out;
        const int sp = vals[s].producer;
        if (sp < 0 || nodes[sp].op != "matmul" || nodes[sp].fused || !sole_use(s, pp)) continue;
        const int t = nodes[sp].in[1], q = nodes[sp].in[0];
        const int tp = vals[t].producer;
        if (tp < 0 || nodes[tp].op != "transpose" || !sole_use(t, sp)) continue;
        if (vals[p].uses.size() != 1 || vals[p].output) continue;
        const int op_ = vals[p].uses[0];
        Node &O = nodes[op_];
        if (O.op != "matmul" || O.in[0] != p || O.in[1] == p) continue;
        const int k = nodes[tp].in[0], v = O.in[1];
        const auto &qd = vals[q].dims, &kd = vals[k].dims, &vd = vals[v].dims;
        if (qd.size() < 2 || qd.size() != kd.size() || kd.size() != vd.size()) continue;
        bool same_batch = true;
        for (size_t i = 0; i + 2 < qd.size(); ++i) same_batch &= qd[i] == kd[i] && kd[i] == vd[i];
        if (!same_batch || qd.back() != kd.back() || kd[kd.size() - 2] != vd[vd.size() - 2]) continue;
        // head dims the attention kernels take (tcgen05: 64 / 128; CUDA cores:
        // up to 256); wider heads run unfused (GEMM, softmax, GEMM)
        if (qd.back() > 256 || vd.back() > 256) continue;
        if (vals[q].dtype != vals[k].dtype || vals[k].dtype != vals[v].dtype) continue;
        const std::vector<int> group = {tp, sp, pp, op_};
        if (!safe_to_defer({q, k, v}, std::min(tp, sp), op_, group)) continue;
        for (int g : group) nodes[g].fused = true;
        vals[t].live = vals[s].live = vals[p].live = false;
        Step st;
        st.kind = K_ATTN;
        st.pos = op_;
        st.a = q; st.b = k; st.c = v; st.out = O.out;
        st.what = "attention (fused transpose, matmul, softmax, matmul)";
        step_at[op_] = (int)steps.size();
        steps.push_back(st);
      }
    }
    // 2. every remaining node, with transposes folded into GEMM operands and
    //    bias / SiLU fused into the GEMM epilogue
    for (int i = 0; i < n_nodes; ++i) {
      Node &n = nodes[i];
      if (n.fused) continue;
      const std::string &op = n.op;
      Step st;
      st.pos = i;
      st.out = n.out;
      if (op == "matmul" || op == "batch_matmul") {
        st.kind = K_GEMM;
        st.a = n.in[0];
        st.b = n.in[1];
        st.what = "gemm";
        int last = i;
        std::vector<int> group = {i};
        if (fuse) {
          // transposed operands: read the transpose's input in the other layout
          for (int side = 0; side < 2; ++side) {
            const int x = side == 0 ? st.a : st.b;
            const int xp = vals[x].producer;
            if (xp < 0 || nodes[xp].op != "transpose" || vals[x].output) continue;
            bool only_gemms = true;
            for (int u : vals[x].uses)
              only_gemms &= nodes[u].op == "matmul" || nodes[u].op == "batch_matmul";
            if (!only_gemms) continue;
            const int src = nodes[xp].in[0];
            if (!safe_to_defer({src}, xp, i, {xp, i})) continue;
            if (side == 0) { st.a = src; st.a_t = 1; } else { st.b = src; st.b_t = 1; }
            st.what += side == 0 ? " A^T" : " B^T";
          }
          // epilogue: add(., bias[N]) then silu
          int cur = n.out;
          const int64_t N = vals[n.out].last();
          if (vals[cur].uses.size() == 1 && !vals[cur].output) {
            Node &A = nodes[vals[cur].uses[0]];
            if (A.op == "add" && A.in.size() == 2 && !A.fused) {
              const int other = A.in[0] == cur ? A.in[1] : A.in[0];
              const int src = other != cur ? bias_source(other, N, vals[cur].uses[0]) : -1;
              const int ap = vals[cur].uses[0];
              if (src >= 0 && vals[src].dtype == vals[cur].dtype &&
                  safe_to_defer({st.a, st.b, src}, i, ap, {i, ap})) {
                st.bias = src;
                group.push_back(ap);
                last = ap;
                A.fused = true;
                // a reshape feeding only this add is not materialised
                if (other != src && vals[other].producer >= 0) {
                  nodes[vals[other].producer].fused = true;
                  vals[other].live = false;
                }
                vals[cur].live = false;
                cur = A.out;
                st.what += " +bias";
              }
            }
          }
          if (vals[cur].uses.size() == 1 && !vals[cur].output) {
            const int sp = vals[cur].uses[0];
            Node &S = nodes[sp];
            if (S.op == "silu" && !S.fused &&
                safe_to_defer({st.a, st.b, st.bias}, i, sp, {i, last, sp})) {
              S.fused = true;
              vals[cur].live = false;
              cur = S.out;
              last = sp;
              st.silu = 1;
              st.what += " +silu";
            }
          }
          // SwiGLU gate: mul(silu(.), U) with U of the output's full shape
          // multiplies in the epilogue (the spec's `swiglu` pattern)
          if (st.silu && vals[cur].uses.size() == 1 && !vals[cur].output) {
            const int mp = vals[cur].uses[0];
            Node &Mu = nodes[mp];
            if (Mu.op == "mul" && Mu.in.size() == 2 && !Mu.fused && Mu.in[0] != Mu.in[1]) {
              const int other = Mu.in[0] == cur ? Mu.in[1] : Mu.in[0];
              const Val &ov = vals[other];
              if (ov.numel() == vals[cur].numel() && ov.last() == N && ov.dtype == vals[cur].dtype &&
                  safe_to_defer({st.a, st.b, st.bias, other}, i, mp, {i, last, mp})) {
                Mu.fused = true;
                vals[cur].live = false;
                cur = Mu.out;
                last = mp;
                st.c = other;
                st.res_mul = 1;
                st.what += " +swiglu";
              }
            }
          }
          // residual: add(., R) with R of the output's full shape, added last
          if (!st.res_mul && vals[cur].uses.size() == 1 && !vals[cur].output) {
            const int rp = vals[cur].uses[0];
            Node &R = nodes[rp];
            if (R.op == "add" && R.in.size() == 2 && !R.fused && R.in[0] != R.in[1]) {
              const int other = R.in[0] == cur ? R.in[1] : R.in[0];
              const Val &ov = vals[other];
              if (ov.numel() == vals[cur].numel() && ov.last() == N && ov.dtype == vals[cur].dtype &&
                  safe_to_defer({st.a, st.b, st.bias, other}, i, rp, {i, last, rp})) {
                R.fused = true;
                vals[cur].live = false;
                cur = R.out;
                last = rp;
                st.c = other;
                st.what += " +residual";
              }
            }
          }
          st.out = cur;
        }
        st.pos = last;
      } else if (op == "transpose") {
        // dropped below if every consumer GEMM reads its source transposed
        st.kind = K_TRANSPOSE;
        st.a = n.in[0];
        st.what = "transpose";
      } else if (op == "softmax") {
        st.kind = K_SOFTMAX; st.a = n.in[0]; st.what = "softmax";
      } else if (op == "rmsnorm") {
        st.kind = K_RMSNORM; st.a = n.in[0];
        st.b = n.in.size() > 1 ? n.in[1] : -1;
        st.c = n.in.size() > 2 ? n.in[2] : -1;
        st.what = "rmsnorm";
      } else if (op == "silu") {
        st.kind = K_UNARY; st.a = n.in[0]; st.op = 1; st.what = "silu";
        // swiglu: mul(silu(x), y) of one shape and dtype -> one pass
        const int so = n.out;
        if (fuse && vals[so].uses.size() == 1 && !vals[so].output) {
          const int mp = vals[so].uses[0];
          Node &Mu = nodes[mp];
          if (Mu.op == "mul" && Mu.in.size() == 2 && !Mu.fused && Mu.in[0] != Mu.in[1]) {
            const int other = Mu.in[0] == so ? Mu.in[1] : Mu.in[0];
            const Val &xv = vals[n.in[0]], &ov = vals[other];
            if (ov.numel() == vals[so].numel() && xv.numel() == ov.numel() &&
                xv.dtype == ov.dtype && ov.dtype == vals[Mu.out].dtype &&
                vals[so].dtype == xv.dtype && safe_to_defer({n.in[0], other}, i, mp, {i, mp})) {
              Mu.fused = true;
              vals[so].live = false;
              st.kind = K_SWIGLU;
              st.b = other;
              st.out = Mu.out;
              st.pos = mp;
              st.what = "swiglu (fused silu, mul)";
            }
          }
        }
      } else if (op == "reshape") {
        st.kind = K_UNARY; st.a = n.in[0]; st.op = 0; st.what = "reshape";
      } else if (op == "add" || op == "sub" || op == "mul" || op == "div") {
        st.kind = K_BINARY;
        st.a = n.in[0];
        st.b = n.in.size() > 1 ? n.in[1] : n.in[0];
        st.op = op == "add" ? 0 : op == "sub" ? 1 : op == "mul" ? 2 : 3;
        st.what = op;
        // residual + norm: rmsnorm(add(a, b)) with a, b of one shape runs as
        // one row kernel at the norm's place; the sum is stored only when
        // something besides the norm reads it (all such reads come after)
        const int h = n.out;
        int rp = -1;
        bool later = true;
        for (int u : vals[h].uses) {
          if (nodes[u].op == "rmsnorm" && !nodes[u].fused && nodes[u].in[0] == h && rp < 0) rp = u;
        }
        for (int u : vals[h].uses)
          if (u != rp && u <= rp) later = false;
        if (fuse && op == "add" && n.in.size() == 2 && rp > i && later) {
          const Node &Rn = nodes[rp];
          const Val &av = vals[n.in[0]], &bv = vals[n.in[1]];
          const int gm = Rn.in.size() > 1 ? Rn.in[1] : -1, bt = Rn.in.size() > 2 ? Rn.in[2] : -1;
          const int C = (int)vals[h].last();
          bool ok = av.numel() == bv.numel() && av.numel() == vals[h].numel() &&
                    av.dtype == bv.dtype && av.dtype == vals[h].dtype &&
                    vals[Rn.out].dtype == av.dtype;
          for (int g : {gm, bt})
            ok = ok && (g < 0 || (vals[g].numel() == C && vals[g].dtype == av.dtype));
          if (ok && safe_to_defer({n.in[0], n.in[1], gm, bt}, i, rp, {i, rp})) {
            nodes[rp].fused = true;
            const bool keep_h = vals[h].output || vals[h].uses.size() > 1;
            if (!keep_h) vals[h].live = false;
            st.kind = K_ADD_RMSNORM;
            st.d = gm;
            st.e = bt;
            st.out = Rn.out;
            st.out2 = keep_h ? h : -1;
            st.pos = rp;
            st.what = keep_h ? "add+rmsnorm (fused residual add and norm, sum stored)"
                             : "add+rmsnorm (fused residual add and norm)";
          }
        }
      } else if (op == "broadcast") {
        st.kind = K_BINARY; st.a = n.in[0]; st.b = n.in[0]; st.op = 4; st.what = "broadcast";
      } else if (op == "silu_grad") {
        st.kind = K_SILU_GRAD; st.a = n.in[0]; st.b = n.in[1]; st.what = "silu_grad";
      } else if (op == "softmax_grad") {
        st.kind = K_SOFTMAX_GRAD; st.a = n.in[0]; st.b = n.in[1]; st.what = "softmax_grad";
      } else if (op == "rmsnorm_grad") {
        st.kind = K_RMSNORM_GRAD; st.a = n.in[0]; st.b = n.in[1]; st.c = n.in[2];
        st.what = "rmsnorm_grad";
      } else if (op == "reduce_sum") {
        st.kind = K_REDUCE; st.a = n.in[0]; st.what = "reduce_sum";
      } else if (op == "permute") {
        // the dump carries no permutation: it is read off the symbolic dims
        // (each output dim names one input dim); the gradient graph records a
        // permute's output unpermuted, which reads as the identity and is
        // refused, as is any ambiguity (the launch plan carries the attribute)
        const Val &x = vals[n.in[0]], &o = vals[n.out];
        st.kind = K_PERMUTE;
        st.a = n.in[0];
        st.what = "permute";
        bool ok = x.sdims.size() == o.sdims.size() && !x.sdims.empty() && x.sdims.size() <= 4;
        bool ident = true;
        for (size_t i = 0; ok && i < o.sdims.size(); ++i) {
          int hit = -1, hits = 0;
          for (size_t j = 0; j < x.sdims.size(); ++j)
            if (x.sdims[j] == o.sdims[i]) {
              hit = (int)j;
              ++hits;
            }
          ok = hits == 1;
          st.perm[i] = hit;
          ident = ident && hit == (int)i;
        }
        if (!ok || ident)
          return fail(BWPP_CUDA_ERR_UNSUPPORTED,
                      "permute (n%d): the permutation cannot be read off the dump's shapes; run "
                      "the compiler's launch plan (bwppc --target cuda)", n.id);
      } else if (op == "reduce_max" || op == "reduce_max_mask") {
        // axis: the dim the forward output keeps as 1 (the graph's default:
        // the last); the mask has the input's shape, so it takes the last
        st.kind = K_REDUCE_MAX;
        st.a = n.in[0];
        st.op = op == "reduce_max" ? 0 : 1;
        st.what = op;
        const auto &xd = vals[n.in[0]].dims, &od = vals[n.out].dims;
        st.axis = (int)xd.size() - 1;
        if (st.op == 0 && od.size() == xd.size())
          for (size_t i = 0; i < xd.size(); ++i)
            if (od[i] == 1 && xd[i] != 1) {
              st.axis = (int)i;
              break;
            }
      } else if (op == "reduce_max_grad") {
        // mask * (dy broadcast to x's shape): elementwise
        st.kind = K_BINARY; st.a = n.in[0]; st.b = n.in[1]; st.op = 2; st.what = "reduce_max_grad";
      } else {
        return fail(BWPP_CUDA_ERR_UNSUPPORTED, "op %s (n%d) is not supported by the executor",
                    op.c_str(), n.id);
      }
      steps.push_back(st);
    }
    // 3. dead steps: a step runs only when its output is a graph output or
    //    read by a step that runs (folded transposes, reshapes of a fused
    //    bias and unused graph branches drop out here)
    std::stable_sort(steps.begin(), steps.end(),
                     [](const Step &x, const Step &y) { return x.pos < y.pos; });
    std::vector<char> need(vals.size(), 0), keep(steps.size(), 0);
    for (int i = (int)steps.size() - 1; i >= 0; --i) {
      const Step &st = steps[i];
      const bool want2 = st.out2 >= 0 && (vals[st.out2].output || need[st.out2]);
      if (!vals[st.out].output && !need[st.out] && !want2) continue;
      keep[i] = 1;
      for (int x : {st.a, st.b, st.c, st.bias, st.d, st.e})
        if (x >= 0) need[x] = 1;
    }
    std::vector<Step> kept;
    for (size_t i = 0; i < steps.size(); ++i) {
      if (keep[i]) {
        kept.push_back(steps[i]);
      } else {
        vals[steps[i].out].live = false;
        if (steps[i].out2 >= 0) vals[steps[i].out2].live = false;
        nodes[steps[i].pos].fused = true;
      }
    }
    steps = kept;
    for (Step &st : steps)
      if (st.kind == K_RMSNORM || st.kind == K_RMSNORM_GRAD || st.kind == K_ADD_RMSNORM) st.eps = eps;
    return BWPP_CUDA_OK;
  }

  // 4. per-step shape checks, binary broadcast modes, reduction axes, aliasing
  // (both plan sources)
  int finish() {
    for (Step &st : steps) {
      if (st.kind == K_PERMUTE) {
        const auto &xd = vals[st.a].dims, &od = vals[st.out].dims;
        bool ok = xd.size() == od.size() && !xd.empty() && xd.size() <= 4;
        std::vector<int> seen(4, 0);
        for (size_t i = 0; ok && i < xd.size(); ++i) {
          const int p = st.perm[i];
          ok = p >= 0 && p < (int)xd.size() && !seen[p]++ && od[i] == xd[p];
        }
        if (!ok) return fail(BWPP_CUDA_ERR_ARG, "permute at n%d: permutation and shapes", nodes[st.pos].id);
      }
      if (st.kind == K_REDUCE_MAX) {
        const auto &xd = vals[st.a].dims;
        if (st.axis < 0 || st.axis >= (int)xd.size())
          return fail(BWPP_CUDA_ERR_ARG, "reduce_max at n%d: axis", nodes[st.pos].id);
        int64_t expect = vals[st.a].numel();
        if (st.op == 0) expect /= xd[st.axis];
        if (vals[st.out].numel() != expect)
          return fail(BWPP_CUDA_ERR_ARG, "reduce_max at n%d: output shape", nodes[st.pos].id);
      }
      Val &o = vals[st.out];
      if (st.kind == K_BINARY) {
        Val *a = &vals[st.a], *b = &vals[st.b];
        if (st.op == 4) {  // broadcast: b -> shape of out
          st.a = st.b;
          a = b;
          const int64_t C = o.last(), R = o.rows();
          st.bmode = b->numel() == o.numel() ? 0 : b->numel() == C ? 1
                   : (b->numel() == R && b->last() == 1) ? 2 : b->numel() == 1 ? 3 : -1;
        } else {
          if (a->numel() < b->numel()) {  // broadcast the first operand
            std::swap(st.a, st.b);
            std::swap(a, b);
            if (st.op == 1) st.op = 5;       // b - a
            else if (st.op == 3) st.op = 6;  // b / a
          }
          if (a->numel() != o.numel())
            return fail(BWPP_CUDA_ERR_UNSUPPORTED, "%s at n%d: operand shapes", st.what.c_str(),
                        nodes[st.pos].id);
          const int64_t C = o.last(), R = o.rows();
          st.bmode = b->numel() == o.numel() ? 0 : b->numel() == C ? 1
                   : (b->numel() == R && b->last() == 1) ? 2 : b->numel() == 1 ? 3 : -1;
        }
        if (st.bmode < 0)
          return fail(BWPP_CUDA_ERR_UNSUPPORTED, "%s at n%d: broadcast pattern", st.what.c_str(),
                      nodes[st.pos].id);
      }
      if (st.kind == K_REDUCE) {
        const auto &xd = vals[st.a].dims;
        if (xd.size() == 2 && o.numel() == xd[1] && xd[0] != 1) st.axis = 0;
        else if (o.numel() == vals[st.a].rows()) st.axis = 1;
        else return fail(BWPP_CUDA_ERR_UNSUPPORTED, "reduce_sum at n%d: axis", nodes[st.pos].id);
      }
      // The memory plan may hand an output the buffer of an input that dies
      // at this node (compiler/mem_plan.c frees inputs before allocating the
      // output).  Row-wise and elementwise kernels run in place; these do
      // not, so their output gets a buffer of its own.
      // (A GEMM's residual is read before the same elements are stored, so
      // it may share the output's buffer.)
      if (st.kind == K_GEMM || st.kind == K_ATTN || st.kind == K_TRANSPOSE || st.kind == K_REDUCE ||
          st.kind == K_PERMUTE || (st.kind == K_REDUCE_MAX && st.op == 0)) {
        for (int x : {st.a, st.b, st.kind == K_GEMM ? -1 : st.c, st.bias})
          if (x >= 0 && !vals[x].input && vals[x].buffer >= 0 && vals[x].buffer == o.buffer)
            o.buffer = -1;
      }
    }
    return BWPP_CUDA_OK;
  }

  // ------------------------------------------------------------------ memory
  size_t gemm_dims(const Step &st, int64_t &M, int64_t &N, int64_t &K, int64_t &batch) const {
    const auto &A = vals[st.a].dims, &B = vals[st.b].dims;
    // A^T is read MN-major from X [K, M]; B^T is read K-major from X [N, K]
    M = st.a_t ? A[A.size() - 1] : A[A.size() - 2];
    K = st.a_t ? A[A.size() - 2] : A[A.size() - 1];
    N = st.b_t ? B[B.size() - 2] : B[B.size() - 1];
    batch = vals[st.out].numel() / std::max<int64_t>(1, M * N);
    return 0;
  }

  int allocate() {
    // bytes per memory-plan buffer (live values only) and per unshared value
    std::vector<size_t> buf_bytes(mp_buffers, 0);
    std::vector<size_t> own(vals.size(), 0);
    for (auto &v : vals) {
      if (v.id < 0 || v.input || !v.live) continue;
      if (!v.known) return fail(BWPP_CUDA_ERR_ARG, "shape of v%d unknown", v.id);
      const size_t bytes = ((size_t)v.numel() * dt_size(v.dtype) + 255) & ~(size_t)255;
      if (v.buffer >= 0) buf_bytes[v.buffer] = std::max(buf_bytes[v.buffer], bytes);
      else own[v.id] = bytes;
    }
    // scratch: aliased outputs, fp32 biases, bf16 operand copies
    size_t scratch = 0, bias_total = 0;
    for (Step &st : steps) {
      size_t need = 0;
      const Val &o = vals[st.out];
      if (st.kind == K_GEMM) {
        if (vals[st.a].dtype == DT_F32 || vals[st.b].dtype != vals[st.a].dtype)
          need += ((size_t)(vals[st.a].numel() + vals[st.b].numel()) * 2 + 512) & ~(size_t)255;
        if (o.dtype == DT_BF16 && vals[st.a].dtype == DT_F16)
          need += ((size_t)o.numel() * 4 + 255) & ~(size_t)255;
        if (st.bias >= 0) {
          st.bias_off = bias_total;
          bias_total += ((size_t)vals[st.bias].numel() * 4 + 255) & ~(size_t)255;
        }
      }
      if (st.kind == K_ATTN) {
        if (vals[st.a].dtype == DT_F32)
          need += ((size_t)(vals[st.a].numel() + vals[st.b].numel() + vals[st.c].numel()) * 2 + 768) &
                  ~(size_t)255;
        if (vals[st.a].dtype != DT_F16) need += ((size_t)o.numel() * 4 + 255) & ~(size_t)255;
      }
      scratch = std::max(scratch, need);
    }
    std::vector<size_t> buf_off(mp_buffers, 0);
    size_t off = 0;
    for (int b = 0; b < mp_buffers; ++b) {
      buf_off[b] = off;
      off += buf_bytes[b];
    }
    std::vector<size_t> own_off(vals.size(), 0);
    for (auto &v : vals)
      if (v.id >= 0 && own[v.id]) {
        own_off[v.id] = off;
        off += own[v.id];
      }
    if (from_launch) {
      // the compiler laid the graph's values out; check its offsets fit
      for (auto &v : vals) {
        if (v.id < 0 || v.input || !v.live) continue;
        const size_t bytes = (size_t)v.numel() * dt_size(v.dtype);
        if (v.off == SIZE_MAX || v.off + bytes > graph_bytes || (v.off & 255))
          return fail(BWPP_CUDA_ERR_ARG, "launch plan: v%d has no valid arena offset", v.id);
      }
      off = graph_bytes;
    }
    const size_t bias_off = off;
    off += bias_total;
    scratch_off = off;
    scratch_bytes = scratch;
    off += scratch;
    arena_bytes = off;
    for (Step &st : steps) st.bias_off += bias_off;
    if (!ctx) return BWPP_CUDA_OK;  // inspection only
    if (arena_bytes) {
      if (cudaMalloc(&arena, arena_bytes) != cudaSuccess) {
        (void)cudaGetLastError();
        arena = nullptr;
        return fail(BWPP_CUDA_ERR_NOMEM, "cudaMalloc of %zu bytes failed", arena_bytes);
      }
    }
    for (auto &v : vals) {
      if (v.id < 0 || v.input || !v.live) continue;
      v.ptr = arena + (from_launch ? v.off : v.buffer >= 0 ? buf_off[v.buffer] : own_off[v.id]);
    }
    return BWPP_CUDA_OK;
  }

  // ------------------------------------------------------------------- run
  int run_step(const Step &st) {
    BwppCudaCtx *c = ctx;
    const Val &o = vals[st.out];
    uint8_t *scratch = arena + scratch_off;
    void *out = o.ptr;
    size_t used = 0;
    auto P = [&](int id) -> void * { return id >= 0 ? vals[id].ptr : nullptr; };
    int rc = BWPP_CUDA_OK;
    switch (st.kind) {
      case K_GEMM: {
        int64_t M, N, K, batch;
        gemm_dims(st, M, N, K, batch);
        const Val &A = vals[st.a], &B = vals[st.b];
        const uint16_t *pa = (const uint16_t *)A.ptr, *pb = (const uint16_t *)B.ptr;
        int ab_f16 = A.dtype == DT_F16 ? 1 : 0;
        if (A.dtype == DT_F32 || B.dtype != A.dtype) {  // round operands to bf16
          uint16_t *ca = (uint16_t *)(scratch + used);
          used += ((size_t)A.numel() * 2 + 255) & ~(size_t)255;
          uint16_t *cb = (uint16_t *)(scratch + used);
          used += ((size_t)B.numel() * 2 + 255) & ~(size_t)255;
          rc = bwpp_plan_convert(c, A.dtype, DT_BF16, A.ptr, ca, A.numel());
          if (!rc) rc = bwpp_plan_convert(c, B.dtype, DT_BF16, B.ptr, cb, B.numel());
          pa = ca;
          pb = cb;
          ab_f16 = 0;
        }
        const float *bias = nullptr;
        if (!rc && st.bias >= 0) {
          const Val &bv = vals[st.bias];
          float *b32 = (float *)(arena + st.bias_off);
          rc = bwpp_plan_convert(c, bv.dtype, DT_F32, bv.ptr, b32, bv.numel());
          bias = b32;
        }
        // output: fp32, or 16-bit of the operand type; bf16 out of f16
        // operands goes through fp32 scratch
        void *dst = out;
        int out16 = o.dtype != DT_F32, out_f16 = o.dtype == DT_F16;
        bool conv_after = false;
        if (o.dtype == DT_BF16 && ab_f16) {
          dst = scratch + used;
          out16 = 0;
          conv_after = true;
        }
        if (o.dtype == DT_F16 && !ab_f16) out_f16 = 1;
        const size_t osz = out16 ? 2 : 4;
        const int64_t a_b = (A.numel() / (M * K) > 1) ? M * K : 0;
        const int64_t b_b = (B.numel() / (K * N) > 1) ? K * N : 0;
        const Val *R = st.c >= 0 ? &vals[st.c] : nullptr;
        const int res16 = (!R ? 0 : R->dtype == DT_F16 ? 2 : R->dtype == DT_BF16 ? 1 : 0) |
                          (st.res_mul ? 4 : 0);
        for (int64_t i = 0; !rc && i < batch; ++i) {
          const void *res = R ? (const uint8_t *)R->ptr + (size_t)(i * M * N) * dt_size(R->dtype)
                              : nullptr;
          rc = bwpp_gemm_launch_dt(c, pa + i * a_b, st.a_t, st.a_t ? (uint32_t)M : (uint32_t)K,
                                   pb + i * b_b, st.b_t ? 0 : 1, st.b_t ? (uint32_t)K : (uint32_t)N,
                                   (uint8_t *)dst + (size_t)(i * M * N) * osz, (uint32_t)N,
                                   (uint32_t)M, (uint32_t)N, (uint32_t)K, bias, st.silu, res,
                                   (uint32_t)N, out16, 0, ab_f16, out_f16, res16);
        }
        launches += batch;
        if (!rc && conv_after) rc = bwpp_plan_convert(c, DT_F32, DT_BF16, dst, out, o.numel());
        break;
      }
      case K_ATTN: {
        const Val &q = vals[st.a], &k = vals[st.b], &v = vals[st.c];
        const int64_t Tq = q.dims[q.dims.size() - 2], D = q.last();
        const int64_t Tk = k.dims[k.dims.size() - 2], Dv = v.last();
        const int64_t BH = q.numel() / (Tq * D);
        const uint16_t *pq = (const uint16_t *)q.ptr, *pk = (const uint16_t *)k.ptr,
                       *pv = (const uint16_t *)v.ptr;
        if (q.dtype == DT_F32) {
          uint16_t *cq = (uint16_t *)(scratch + used);
          used += ((size_t)q.numel() * 2 + 255) & ~(size_t)255;
          uint16_t *ck = (uint16_t *)(scratch + used);
          used += ((size_t)k.numel() * 2 + 255) & ~(size_t)255;
          uint16_t *cv = (uint16_t *)(scratch + used);
          used += ((size_t)v.numel() * 2 + 255) & ~(size_t)255;
          rc = bwpp_plan_convert(c, DT_F32, DT_BF16, q.ptr, cq, q.numel());
          if (!rc) rc = bwpp_plan_convert(c, DT_F32, DT_BF16, k.ptr, ck, k.numel());
          if (!rc) rc = bwpp_plan_convert(c, DT_F32, DT_BF16, v.ptr, cv, v.numel());
          pq = cq; pk = ck; pv = cv;
        }
        const int f16 = q.dtype == DT_F16;
        void *dst = out;
        if (!f16 && o.dtype != DT_F32) {
          dst = scratch + used;
        }
        if (!rc)
          rc = bwpp_attention_launch(c, pq, pk, pv, dst, (uint32_t)BH, (uint32_t)Tq, (uint32_t)Tk,
                                     (uint32_t)D, (uint32_t)Dv, (uint64_t)(Tq * D), (uint64_t)(Tk * D),
                                     (uint64_t)(Tk * Dv), (uint64_t)(Tq * Dv), (uint32_t)D,
                                     (uint32_t)D, (uint32_t)Dv, (uint32_t)Dv, 1.0f, 0, f16);
        ++launches;
        if (!rc && dst != out) rc = bwpp_plan_convert(c, DT_F32, o.dtype, dst, out, o.numel());
        break;
      }
      case K_SOFTMAX: {
        const Val &x = vals[st.a];
        const uint32_t R = (uint32_t)x.rows(), C = (uint32_t)x.last();
        if (x.dtype == DT_F16) rc = bwpp_cuda_softmax_f16(c, (const uint16_t *)x.ptr, (uint16_t *)out, R, C, C);
        else if (x.dtype == DT_F32) rc = bwpp_cuda_softmax_fwd_f32(c, (const float *)x.ptr, (float *)out, R, C, C);
        else rc = bwpp_plan_softmax(c, x.dtype, x.ptr, out, R, C);
        ++launches;
        break;
      }
      case K_RMSNORM: {
        const Val &x = vals[st.a];
        const uint32_t R = (uint32_t)x.rows(), C = (uint32_t)x.last();
        if (x.dtype == DT_F16)
          rc = bwpp_cuda_rmsnorm_f16(c, (const uint16_t *)x.ptr, (uint16_t *)out,
                                     (const uint16_t *)P(st.b), (const uint16_t *)P(st.c), R, C, C, st.eps);
        else if (x.dtype == DT_F32)
          rc = bwpp_cuda_rmsnorm_fwd_f32(c, (const float *)x.ptr, (float *)out, (const float *)P(st.b),
                                         (const float *)P(st.c), R, C, C, st.eps);
        else rc = bwpp_plan_rmsnorm(c, x.dtype, x.ptr, P(st.b), P(st.c), out, R, C, st.eps);
        ++launches;
        break;
      }
      case K_UNARY:
        if (st.op == 0 && out == vals[st.a].ptr) break;  // reshape in place: nothing to do
        rc = bwpp_plan_unary(c, o.dtype, vals[st.a].ptr, out, o.numel(), st.op);
        ++launches;
        break;
      case K_BINARY:
        rc = bwpp_plan_binary(c, o.dtype, vals[st.a].ptr, vals[st.b].ptr, out, (uint32_t)o.rows(),
                              (uint32_t)o.last(), st.op, st.bmode);
        ++launches;
        break;
      case K_TRANSPOSE: {
        const Val &x = vals[st.a];
        const int64_t R = x.dims[x.dims.size() - 2], C = x.last();
        rc = bwpp_plan_transpose(c, x.dtype, x.ptr, out, (uint32_t)(x.numel() / (R * C)),
                                 (uint32_t)R, (uint32_t)C);
        ++launches;
        break;
      }
      case K_SILU_GRAD:
        rc = bwpp_plan_silu_grad(c, o.dtype, vals[st.a].ptr, vals[st.b].ptr, out, o.numel());
        ++launches;
        break;
      case K_SOFTMAX_GRAD:
        rc = bwpp_plan_softmax_grad(c, o.dtype, vals[st.a].ptr, vals[st.b].ptr, out,
                                    (uint32_t)o.rows(), (uint32_t)o.last());
        ++launches;
        break;
      case K_RMSNORM_GRAD:
        rc = bwpp_plan_rmsnorm_grad(c, o.dtype, vals[st.a].ptr, vals[st.b].ptr, vals[st.c].ptr, out,
                                    (uint32_t)o.rows(), (uint32_t)o.last(), st.eps);
        ++launches;
        break;
      case K_PERMUTE: {
        const Val &x = vals[st.a];
        rc = bwpp_plan_permute(c, x.dtype, x.ptr, out, (int)x.dims.size(), x.dims.data(), st.perm);
        ++launches;
        break;
      }
      case K_REDUCE_MAX: {
        const Val &x = vals[st.a];
        int64_t outer = 1, inner = 1;
        for (int i = 0; i < st.axis; ++i) outer *= x.dims[i];
        for (size_t i = st.axis + 1; i < x.dims.size(); ++i) inner *= x.dims[i];
        rc = bwpp_plan_reduce_max(c, x.dtype, x.ptr, out, (uint32_t)outer, (uint32_t)x.dims[st.axis],
                                  (uint32_t)inner, st.op);
        ++launches;
        break;
      }
      case K_SWIGLU:
        rc = bwpp_plan_swiglu(c, o.dtype, vals[st.a].ptr, vals[st.b].ptr, out, o.numel());
        ++launches;
        break;
      case K_ADD_RMSNORM:
        rc = bwpp_plan_add_rmsnorm(c, o.dtype, vals[st.a].ptr, vals[st.b].ptr, P(st.d), P(st.e),
                                   st.out2 >= 0 ? vals[st.out2].ptr : nullptr, out,
                                   (uint32_t)o.rows(), (uint32_t)o.last(), st.eps);
        ++launches;
        break;
      case K_REDUCE: {
        const Val &x = vals[st.a];
        const uint32_t R = st.axis == 0 ? (uint32_t)x.dims[0] : (uint32_t)x.rows();
        const uint32_t C = st.axis == 0 ? (uint32_t)x.dims[1] : (uint32_t)x.last();
        rc = bwpp_plan_reduce_sum(c, x.dtype, x.ptr, out, R, C, st.axis);
        ++launches;
        break;
      }
    }
    return rc;
  }

  int run() {
    if (!ctx) return fail(BWPP_CUDA_ERR_ARG, "plan was created without a context (inspection only)");
    int rc = bwpp_ctx_enter(ctx);
    if (rc) return rc;
    for (auto &v : vals)
      if (v.id >= 0 && v.input && !v.ptr && !v.uses.empty())
        return fail(BWPP_CUDA_ERR_ARG, "input v%d (%s) is not bound", v.id, v.name.c_str());
    launches = 0;
    for (const Step &st : steps) {
      rc = run_step(st);
      if (rc) return rc;
    }
    return BWPP_CUDA_OK;
  }
};

extern "C" {

int bwpp_cuda_plan_create(BwppCudaCtx *ctx, const char *graph_dot, const char *mem_plan,
                          const char *dims, const char *options, BwppCudaPlan **out) {
  if (!out || !graph_dot) return BWPP_CUDA_ERR_ARG;
  *out = nullptr;
  if (ctx) {
    int rc = bwpp_ctx_enter(ctx);
    if (rc) return rc;
  }
  BwppCudaPlan *p = new (std::nothrow) BwppCudaPlan();
  if (!p) return BWPP_CUDA_ERR_NOMEM;
  p->ctx = ctx;
  int rc = p->parse_options(options);
  if (!rc) rc = p->parse_dims(dims);
  if (!rc) rc = p->parse_graph(graph_dot);
  if (!rc && mem_plan) rc = p->parse_mem_plan(mem_plan);
  for (auto &v : p->vals)
    if (!rc && v.id >= 0) rc = p->resolve(v);
  for (auto &n : p->nodes)
    if (!rc) rc = p->infer(n);
  if (!rc) rc = p->lower();
  if (!rc) rc = p->finish();
  if (!rc) rc = p->allocate();
  if (rc) {
    if (p->arena) cudaFree(p->arena);
    delete p;
    return rc;
  }
  tl_err[0] = 0;
  *out = p;
  return BWPP_CUDA_OK;
}

int bwpp_cuda_plan_create_launch(BwppCudaCtx *ctx, const char *launch_plan, const char *options,
                                 BwppCudaPlan **out) {
  if (!out || !launch_plan) return BWPP_CUDA_ERR_ARG;
  *out = nullptr;
  if (ctx) {
    int rc = bwpp_ctx_enter(ctx);
    if (rc) return rc;
  }
  BwppCudaPlan *p = new (std::nothrow) BwppCudaPlan();
  if (!p) return BWPP_CUDA_ERR_NOMEM;
  p->ctx = ctx;
  int rc = p->parse_options(options);
  if (!rc) rc = p->parse_launch(launch_plan);
  if (!rc) rc = p->finish();
  if (!rc) rc = p->allocate();
  if (rc) {
    if (p->arena) cudaFree(p->arena);
    delete p;
    return rc;
  }
  tl_err[0] = 0;
  *out = p;
  return BWPP_CUDA_OK;
}

const char *bwpp_cuda_plan_last_error(void) { return tl_err; }

int bwpp_cuda_plan_describe(const BwppCudaPlan *p, char *buf, size_t len) {
  if (!p) return -1;
  std::string s;
  char line[512];
  for (size_t i = 0; i < p->steps.size(); ++i) {
    const Step &st = p->steps[i];
    const Val &o = p->vals[st.out];
    std::string shp;
    for (size_t d = 0; d < o.dims.size(); ++d) shp += (d ? "," : "") + std::to_string(o.dims[d]);
    snprintf(line, sizeof(line), "%zu n%d %s -> v%d %s [%s]%s\n", i, p->nodes[st.pos].id,
             st.what.c_str(), st.out, dt_name(o.dtype), shp.c_str(),
             o.buffer < 0 && !o.input ? " (own buffer)" : "");
    s += line;
  }
  snprintf(line, sizeof(line), "arena %zu bytes\n", p->arena_bytes);
  s += line;
  if (buf && len) {
    const size_t n = std::min(len - 1, s.size());
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return (int)s.size() + 1;
}

int bwpp_cuda_plan_find(const BwppCudaPlan *p, const char *name) {
  if (!p || !name) return -1;
  for (const auto &v : p->vals)
    if (v.id >= 0 && v.name == name) return v.id;
  return -1;
}

int bwpp_cuda_plan_value_count(const BwppCudaPlan *p) { return p ? (int)p->vals.size() : 0; }

int bwpp_cuda_plan_value_info(const BwppCudaPlan *p, int id, int *dtype, int *rank, int64_t *dims8,
                              int *flags) {
  if (!p || id < 0 || id >= (int)p->vals.size() || p->vals[id].id < 0) return BWPP_CUDA_ERR_ARG;
  const Val &v = p->vals[id];
  if (dtype) *dtype = v.dtype;
  if (rank) *rank = (int)v.dims.size();
  if (dims8)
    for (size_t i = 0; i < v.dims.size() && i < 8; ++i) dims8[i] = v.dims[i];
  if (flags) *flags = (v.input ? 1 : 0) | (v.output ? 2 : 0) | (v.live && !v.input ? 4 : 0);
  return BWPP_CUDA_OK;
}

int bwpp_cuda_plan_bind(BwppCudaPlan *p, int id, void *dev_ptr) {
  if (!p || id < 0 || id >= (int)p->vals.size() || p->vals[id].id < 0 || !dev_ptr)
    return BWPP_CUDA_ERR_ARG;
  Val &v = p->vals[id];
  if (!v.input && !v.output) return p->fail(BWPP_CUDA_ERR_ARG, "v%d is neither input nor output", id);
  // an output bound here is written to the caller's memory instead of its
  // memory-plan buffer (the buffer stays in use by the other values in it)
  v.ptr = dev_ptr;
  v.bound = true;
  return BWPP_CUDA_OK;
}

void *bwpp_cuda_plan_value_ptr(const BwppCudaPlan *p, int id) {
  if (!p || id < 0 || id >= (int)p->vals.size() || p->vals[id].id < 0) return nullptr;
  return p->vals[id].ptr;
}

int bwpp_cuda_plan_run(BwppCudaPlan *p) { return p ? p->run() : BWPP_CUDA_ERR_ARG; }

size_t bwpp_cuda_plan_launches(const BwppCudaPlan *p) { return p ? p->launches : 0; }

int bwpp_cuda_plan_destroy(BwppCudaPlan *p) {
  if (!p) return BWPP_CUDA_ERR_ARG;
  if (p->arena) {
    if (p->ctx) cudaSetDevice(p->ctx->device);
    cudaFree(p->arena);
  }
  delete p;
  return BWPP_CUDA_OK;
}

}  // extern "C"
