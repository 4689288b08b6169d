/* `bwppc --target cuda`: lowers the compiler's graph (compiler/graph_ir.h)
 * to a launch plan for the B200 runtime (runtime/cuda/plan.cu runs it).
 * See codegen_cuda.h for the format.  Plain C11; it reads the graph, the IR
 * and the memory plan through the compiler's public headers only.
 *
 * Steps, once per compile:
 *   1. bind every symbolic dim (--dims) and infer the shapes the graph
 *      leaves rank-unknown (rank-4 matmuls, transposes);
 *   2. fuse: attention (transpose(k) -> matmul(q, .) -> softmax ->
 *      matmul(., v), every intermediate single-use, head dims <= 256);
 *      a transpose read only by matmuls folds into the GEMM operand layout;
 *      the GEMM epilogue takes add(., bias[N] or reshape(bias)) -> silu ->
 *      mul(., U) (the SwiGLU gate) or add(., R) (a residual);
 *      mul(silu(x), y) becomes one swiglu pass; rmsnorm(add(a, b)) one
 *      residual + norm row pass (the sum stored only when read again);
 *      every other node is one launch (permute carries its axes, reduce_max
 *      and its mask their axis, from the graph's attributes);
 *   3. drop launches whose results nobody reads;
 *   4. lay out memory: the memory plan's buffers (only values that are
 *      still materialised count towards a buffer's size), values without a
 *      buffer, and outputs of GEMM / attention / transpose / reductions that
 *      the plan would put in one of their inputs' buffers (those kernels do
 *      not run in place) get storage of their own.
 * A fusion whose deferred inputs the memory plan hands to another value
 * before the fused launch runs is not taken. */
#include "codegen_cuda.h"

#include <ctype.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "mem_plan.h"

enum { DT_F16 = 0, DT_BF16 = 1, DT_F32 = 2 };

enum {
  K_GEMM, K_ATTN, K_SOFTMAX, K_RMSNORM, K_UNARY, K_BINARY, K_TRANSPOSE, K_SILU_GRAD,
  K_SOFTMAX_GRAD, K_RMSNORM_GRAD, K_REDUCE, K_SWIGLU, K_ADD_RMSNORM, K_PERMUTE, K_REDUCE_MAX
};

typedef struct {
  int64_t dims[BWPP_GRAPH_MAX_DIMS];
  int rank, known;
  int dtype, input, output;
  int producer;       /* node position, -1 for graph inputs */
  int *uses;          /* node positions, one per input edge */
  int nuses, cap;
  int buffer;         /* memory-plan buffer, -1: none */
  int live;           /* 0: fused away, never materialised */
  size_t offset;      /* arena offset when materialised */
} CgVal;

typedef struct {
  BwppGraphOpKind op;
  int in[BWPP_GRAPH_MAX_INPUTS];
  int nin, out, fused;
  float eps;
  int axis;                       /* reduce_max (-1: the last) */
  int perm[BWPP_GRAPH_MAX_DIMS];  /* permute */
  int perm_rank;
} CgNode;

typedef struct {
  int kind, pos;
  int a, b, c, out, bias, d, e, out2;
  int a_t, b_t, silu, res_mul, op;
  float eps;
  int axis;
  int perm[BWPP_GRAPH_MAX_DIMS];
  const char *what;
} CgStep;

typedef struct {
  const BwppGraph *g;
  CgVal *v;
  int nv;
  CgNode *n;
  int nn;
  CgStep *s;
  int ns, scap;
  char dim_name[32][32];
  int64_t dim_val[32];
  int ndims;
  int nbuf;
  size_t *buf_bytes, *buf_off;
  size_t arena;
  char err[512];
} Cg;

static BwppStatus cg_fail(Cg *cg, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(cg->err, sizeof(cg->err), fmt, ap);
  va_end(ap);
  return BWPP_ERR;
}

static const char *op_name(BwppGraphOpKind op) {
  static const char *names[] = {
      "matmul", "batch_matmul", "transpose", "permute", "reshape", "broadcast", "add", "sub",
      "mul", "div", "reduce_sum", "reduce_max", "reduce_max_mask", "reduce_max_grad", "softmax",
      "rmsnorm", "silu", "silu_grad", "softmax_grad", "rmsnorm_grad"};
  return (unsigned)op < sizeof(names) / sizeof(names[0]) ? names[op] : "unknown";
}

static const char *dt_name(int dt) { return dt == DT_F16 ? "f16" : dt == DT_BF16 ? "bf16" : "f32"; }
static size_t dt_size(int dt) { return dt == DT_F32 ? 4 : 2; }

static int64_t numel(const CgVal *x) {
  int64_t n = 1;
  for (int i = 0; i < x->rank; ++i) n *= x->dims[i];
  return n;
}
static int64_t last_dim(const CgVal *x) { return x->rank ? x->dims[x->rank - 1] : 1; }

static int is_gemm(BwppGraphOpKind op) {
  return op == BWPP_GOP_MATMUL || op == BWPP_GOP_BATCH_MATMUL;
}

static int add_use(CgVal *x, int pos) {
  if (x->nuses == x->cap) {
    int cap = x->cap ? 2 * x->cap : 4;
    int *u = (int *)realloc(x->uses, (size_t)cap * sizeof(int));
    if (!u) return 0;
    x->uses = u;
    x->cap = cap;
  }
  x->uses[x->nuses++] = pos;
  return 1;
}

/* ---- 1. dims and shapes ------------------------------------------------- */

static BwppStatus parse_dims(Cg *cg, const char *spec) {
  if (!spec || !*spec) return cg_fail(cg, "--target cuda needs --dims NAME=VALUE,... (shapes are static)");
  const char *p = spec;
  while (*p) {
    while (*p == ',' || isspace((unsigned char)*p)) ++p;
    if (!*p) break;
    const char *eq = strchr(p, '=');
    const char *end = strchr(p, ',');
    if (!end) end = p + strlen(p);
    if (!eq || eq > end || eq == p || eq - p >= 32)
      return cg_fail(cg, "--dims: '%.*s' is not NAME=VALUE", (int)(end - p), p);
    if (cg->ndims == 32) return cg_fail(cg, "--dims: more than 32 names");
    memcpy(cg->dim_name[cg->ndims], p, (size_t)(eq - p));
    cg->dim_name[cg->ndims][eq - p] = 0;
    const long long n = atoll(eq + 1);
    if (n <= 0) return cg_fail(cg, "--dims: %s must be positive", cg->dim_name[cg->ndims]);
    cg->dim_val[cg->ndims++] = n;
    p = end;
  }
  return BWPP_OK;
}

static BwppStatus resolve(Cg *cg, int id) {
  const BwppGraphValue *gv = &cg->g->values[id];
  CgVal *x = &cg->v[id];
  if (gv->shape.rank == 0) return BWPP_OK; /* rank unknown: inferred from its producer */
  x->rank = (int)gv->shape.rank;
  for (uint32_t i = 0; i < gv->shape.rank; ++i) {
    const BwppStr d = gv->shape.dims[i];
    if (d.len && isdigit((unsigned char)d.ptr[0])) {
      x->dims[i] = atoll(d.ptr);
      continue;
    }
    int k = 0;
    while (k < cg->ndims && !(strlen(cg->dim_name[k]) == d.len &&
                              strncmp(cg->dim_name[k], d.ptr, d.len) == 0))
      ++k;
    if (k == cg->ndims) return cg_fail(cg, "dim %.*s of v%d is not bound by --dims", (int)d.len, d.ptr, id);
    x->dims[i] = cg->dim_val[k];
  }
  x->known = 1;
  return BWPP_OK;
}

static BwppStatus infer(Cg *cg, int pos) {
  const CgNode *n = &cg->n[pos];
  CgVal *o = &cg->v[n->out];
  int64_t d[BWPP_GRAPH_MAX_DIMS];
  int rank = 0;
  for (int i = 0; i < n->nin; ++i)
    if (!cg->v[n->in[i]].known) return cg_fail(cg, "shape of v%d unknown at n%d", n->in[i], pos);
  const CgVal *A = n->nin > 0 ? &cg->v[n->in[0]] : NULL;
  const CgVal *B = n->nin > 1 ? &cg->v[n->in[1]] : NULL;
  switch (n->op) {
    case BWPP_GOP_MATMUL:
    case BWPP_GOP_BATCH_MATMUL: {
      if (n->nin != 2 || A->rank < 2 || B->rank < 2)
        return cg_fail(cg, "n%d: matmul needs two operands of rank >= 2", pos);
      if (A->dims[A->rank - 1] != B->dims[B->rank - 2])
        return cg_fail(cg, "n%d: matmul inner dims %lld vs %lld", pos,
                       (long long)A->dims[A->rank - 1], (long long)B->dims[B->rank - 2]);
      const CgVal *w = A->rank >= B->rank ? A : B;
      rank = w->rank;
      memcpy(d, w->dims, sizeof(d));
      d[rank - 2] = A->dims[A->rank - 2];
      d[rank - 1] = B->dims[B->rank - 1];
      break;
    }
    case BWPP_GOP_TRANSPOSE: {
      if (A->rank < 2) return cg_fail(cg, "n%d: transpose of rank < 2", pos);
      rank = A->rank;
      memcpy(d, A->dims, sizeof(d));
      const int64_t t = d[rank - 1];
      d[rank - 1] = d[rank - 2];
      d[rank - 2] = t;
      break;
    }
    case BWPP_GOP_SOFTMAX: case BWPP_GOP_SILU: case BWPP_GOP_RMSNORM: case BWPP_GOP_SILU_GRAD:
    case BWPP_GOP_SOFTMAX_GRAD: case BWPP_GOP_RMSNORM_GRAD: case BWPP_GOP_REDUCE_MAX_MASK:
    case BWPP_GOP_REDUCE_MAX_GRAD:
      rank = A->rank;
      memcpy(d, A->dims, sizeof(d));
      break;
    case BWPP_GOP_PERMUTE:
      /* output dim i is input dim perm[i] (the gradient graph records an
       * inverse permute's output unpermuted; this shape wins) */
      if (n->perm_rank != A->rank) return cg_fail(cg, "n%d: permute of rank %d by %d axes", pos, A->rank, n->perm_rank);
      rank = A->rank;
      for (int i = 0; i < rank; ++i) {
        if (n->perm[i] < 0 || n->perm[i] >= rank) return cg_fail(cg, "n%d: permute axis", pos);
        d[i] = A->dims[n->perm[i]];
      }
      break;
    case BWPP_GOP_ADD: case BWPP_GOP_SUB: case BWPP_GOP_MUL: case BWPP_GOP_DIV: {
      const CgVal *w = (!B || numel(A) >= numel(B)) ? A : B;
      rank = w->rank;
      memcpy(d, w->dims, sizeof(d));
      break;
    }
    case BWPP_GOP_REDUCE_SUM:
      if (o->known) return BWPP_OK; /* the axis follows from the output shape */
      rank = A->rank;
      memcpy(d, A->dims, sizeof(d));
      if (rank) d[rank - 1] = 1;
      break;
    default:
      if (!o->known) return cg_fail(cg, "n%d: cannot infer the shape of %s", pos, op_name(n->op));
      return BWPP_OK;
  }
  if (o->known) {
    int64_t a = 1;
    for (int i = 0; i < rank; ++i) a *= d[i];
    if (a != numel(o))
      return cg_fail(cg, "n%d (%s): output v%d has %lld elements, inferred %lld", pos,
                     op_name(n->op), n->out, (long long)numel(o), (long long)a);
    /* the graph records some outputs untransposed (rank-4 transpose): the
     * shape that follows from the operation wins */
    if (n->op != BWPP_GOP_TRANSPOSE && n->op != BWPP_GOP_PERMUTE && !is_gemm(n->op)) return BWPP_OK;
  }
  o->rank = rank;
  memcpy(o->dims, d, sizeof(d));
  o->known = 1;
  return BWPP_OK;
}

/* ---- 2. fusion ---------------------------------------------------------- */

static int sole_use(const Cg *cg, int v, int pos) {
  const CgVal *x = &cg->v[v];
  return !x->output && x->nuses == 1 && x->uses[0] == pos;
}

static int in_group(const int *group, int ng, int j) {
  for (int i = 0; i < ng; ++i)
    if (group[i] == j) return 1;
  return 0;
}

/* Running a launch at `at` that reads `inputs` instead of their readers from
 * `from` on is safe when no node in [from, at) outside `group` writes a
 * buffer one of them lives in. */
static int safe_to_defer(const Cg *cg, const int *inputs, int ni, int from, int at,
                         const int *group, int ng) {
  for (int k = 0; k < ni; ++k) {
    const int x = inputs[k];
    if (x < 0) continue;
    const CgVal *v = &cg->v[x];
    if (v->input || v->buffer < 0) continue;
    for (int j = from; j < at; ++j) {
      if (in_group(group, ng, j) || j == v->producer) continue;
      const int w = cg->n[j].out;
      if (cg->v[w].buffer == v->buffer && w != x) return 0;
    }
  }
  return 1;
}

/* The rank-1 bias behind an add operand: N elements, directly or through
 * reshapes that only feed this add. */
static int bias_source(const Cg *cg, int v, int64_t N, int add_pos) {
  const CgVal *b = &cg->v[v];
  if (numel(b) != N || b->rank > 2 || (b->rank == 2 && b->dims[0] != 1)) return -1;
  int src = v;
  while (cg->v[src].producer >= 0 && cg->n[cg->v[src].producer].op == BWPP_GOP_RESHAPE &&
         sole_use(cg, src, src == v ? add_pos : -2)) {
    src = cg->n[cg->v[src].producer].in[0];
    if (numel(&cg->v[src]) != N) return -1;
  }
  return src;
}

static CgStep *new_step(Cg *cg, int kind, int pos, int out, const char *what) {
  if (cg->ns == cg->scap) {
    int cap = cg->scap ? 2 * cg->scap : 32;
    CgStep *s = (CgStep *)realloc(cg->s, (size_t)cap * sizeof(CgStep));
    if (!s) return NULL;
    cg->s = s;
    cg->scap = cap;
  }
  CgStep *st = &cg->s[cg->ns++];
  memset(st, 0, sizeof(*st));
  st->kind = kind;
  st->pos = pos;
  st->out = out;
  st->a = st->b = st->c = st->bias = st->d = st->e = st->out2 = -1;
  st->eps = 1e-5f;
  st->what = what;
  return st;
}

static BwppStatus fuse_attention(Cg *cg) {
  for (int pp = 0; pp < cg->nn; ++pp) {
    CgNode *P = &cg->n[pp];
    if (P->op != BWPP_GOP_SOFTMAX || P->fused || P->nin != 1) continue;
    const int s = P->in[0], p = P->out;
    const int sp = cg->v[s].producer;
    if (sp < 0 || cg->n[sp].op != BWPP_GOP_MATMUL || cg->n[sp].fused || !sole_use(cg, s, pp)) continue;
    const int t = cg->n[sp].in[1], q = cg->n[sp].in[0];
    const int tp = cg->v[t].producer;
    if (tp < 0 || cg->n[tp].op != BWPP_GOP_TRANSPOSE || !sole_use(cg, t, sp)) continue;
    if (cg->v[p].nuses != 1 || cg->v[p].output) continue;
    const int opos = cg->v[p].uses[0];
    CgNode *O = &cg->n[opos];
    if (O->op != BWPP_GOP_MATMUL || O->in[0] != p || O->in[1] == p) continue;
    const int k = cg->n[tp].in[0], v = O->in[1];
    const CgVal *Q = &cg->v[q], *K = &cg->v[k], *V = &cg->v[v];
    if (Q->rank < 2 || Q->rank != K->rank || K->rank != V->rank) continue;
    int same = 1;
    for (int i = 0; i + 2 < Q->rank; ++i) same &= Q->dims[i] == K->dims[i] && K->dims[i] == V->dims[i];
    if (!same || last_dim(Q) != last_dim(K) || K->dims[K->rank - 2] != V->dims[V->rank - 2]) continue;
    /* head dims the attention kernels take (tcgen05: 64 / 128; CUDA cores:
     * up to 256); wider heads run unfused */
    if (last_dim(Q) > 256 || last_dim(V) > 256) continue;
    if (Q->dtype != K->dtype || K->dtype != V->dtype) continue;
    const int group[4] = {tp, sp, pp, opos};
    const int ins[3] = {q, k, v};
    if (!safe_to_defer(cg, ins, 3, tp < sp ? tp : sp, opos, group, 4)) continue;
    for (int g = 0; g < 4; ++g) cg->n[group[g]].fused = 1;
    cg->v[t].live = cg->v[s].live = cg->v[p].live = 0;
    CgStep *st = new_step(cg, K_ATTN, opos, O->out, "attention");
    if (!st) return cg_fail(cg, "out of memory");
    st->a = q;
    st->b = k;
    st->c = v;
  }
  return BWPP_OK;
}

static BwppStatus lower_gemm(Cg *cg, int i) {
  CgNode *n = &cg->n[i];
  CgStep *st = new_step(cg, K_GEMM, i, n->out, "gemm");
  if (!st) return cg_fail(cg, "out of memory");
  st->a = n->in[0];
  st->b = n->in[1];
  int last = i;
  /* transposed operands: read the transpose's input in the other layout */
  for (int side = 0; side < 2; ++side) {
    const int x = side == 0 ? st->a : st->b;
    const int xp = cg->v[x].producer;
    if (xp < 0 || cg->n[xp].op != BWPP_GOP_TRANSPOSE || cg->v[x].output) continue;
    int only = 1;
    for (int u = 0; u < cg->v[x].nuses; ++u) only &= is_gemm(cg->n[cg->v[x].uses[u]].op);
    if (!only) continue;
    const int src = cg->n[xp].in[0];
    const int grp[2] = {xp, i};
    if (!safe_to_defer(cg, &src, 1, xp, i, grp, 2)) continue;
    if (side == 0) {
      st->a = src;
      st->a_t = 1;
    } else {
      st->b = src;
      st->b_t = 1;
    }
  }
  /* epilogue: add(., bias[N]), then silu, then mul(., U) or add(., R) */
  int cur = n->out;
  const int64_t N = last_dim(&cg->v[n->out]);
  if (cg->v[cur].nuses == 1 && !cg->v[cur].output) {
    const int ap = cg->v[cur].uses[0];
    CgNode *A = &cg->n[ap];
    if (A->op == BWPP_GOP_ADD && A->nin == 2 && !A->fused) {
      const int other = A->in[0] == cur ? A->in[1] : A->in[0];
      const int src = other != cur ? bias_source(cg, other, N, ap) : -1;
      const int ins[3] = {st->a, st->b, src};
      const int grp[2] = {i, ap};
      if (src >= 0 && cg->v[src].dtype == cg->v[cur].dtype && safe_to_defer(cg, ins, 3, i, ap, grp, 2)) {
        st->bias = src;
        last = ap;
        A->fused = 1;
        if (other != src && cg->v[other].producer >= 0) { /* a reshape feeding only this add */
          cg->n[cg->v[other].producer].fused = 1;
          cg->v[other].live = 0;
        }
        cg->v[cur].live = 0;
        cur = A->out;
      }
    }
  }
  if (cg->v[cur].nuses == 1 && !cg->v[cur].output) {
    const int sp = cg->v[cur].uses[0];
    CgNode *S = &cg->n[sp];
    const int ins[3] = {st->a, st->b, st->bias};
    const int grp[3] = {i, last, sp};
    if (S->op == BWPP_GOP_SILU && !S->fused && safe_to_defer(cg, ins, 3, i, sp, grp, 3)) {
      S->fused = 1;
      cg->v[cur].live = 0;
      cur = S->out;
      last = sp;
      st->silu = 1;
    }
  }
  if (st->silu && cg->v[cur].nuses == 1 && !cg->v[cur].output) {
    const int mp = cg->v[cur].uses[0];
    CgNode *Mu = &cg->n[mp];
    if (Mu->op == BWPP_GOP_MUL && Mu->nin == 2 && !Mu->fused && Mu->in[0] != Mu->in[1]) {
      const int other = Mu->in[0] == cur ? Mu->in[1] : Mu->in[0];
      const CgVal *ov = &cg->v[other];
      const int ins[4] = {st->a, st->b, st->bias, other};
      const int grp[3] = {i, last, mp};
      if (numel(ov) == numel(&cg->v[cur]) && last_dim(ov) == N && ov->dtype == cg->v[cur].dtype &&
          safe_to_defer(cg, ins, 4, i, mp, grp, 3)) {
        Mu->fused = 1;
        cg->v[cur].live = 0;
        cur = Mu->out;
        last = mp;
        st->c = other;
        st->res_mul = 1;
      }
    }
  }
  if (!st->res_mul && cg->v[cur].nuses == 1 && !cg->v[cur].output) {
    const int rp = cg->v[cur].uses[0];
    CgNode *R = &cg->n[rp];
    if (R->op == BWPP_GOP_ADD && R->nin == 2 && !R->fused && R->in[0] != R->in[1]) {
      const int other = R->in[0] == cur ? R->in[1] : R->in[0];
      const CgVal *ov = &cg->v[other];
      const int ins[4] = {st->a, st->b, st->bias, other};
      const int grp[3] = {i, last, rp};
      if (numel(ov) == numel(&cg->v[cur]) && last_dim(ov) == N && ov->dtype == cg->v[cur].dtype &&
          safe_to_defer(cg, ins, 4, i, rp, grp, 3)) {
        R->fused = 1;
        cg->v[cur].live = 0;
        cur = R->out;
        last = rp;
        st->c = other;
      }
    }
  }
  st->out = cur;
  st->pos = last;
  return BWPP_OK;
}

/* mul(silu(x), y), one shape and dtype: one swiglu pass at the mul's place */
static int try_swiglu(Cg *cg, int i, CgStep *st) {
  CgNode *n = &cg->n[i];
  const int so = n->out;
  if (cg->v[so].nuses != 1 || cg->v[so].output) return 0;
  const int mp = cg->v[so].uses[0];
  CgNode *Mu = &cg->n[mp];
  if (Mu->op != BWPP_GOP_MUL || Mu->nin != 2 || Mu->fused || Mu->in[0] == Mu->in[1]) return 0;
  const int other = Mu->in[0] == so ? Mu->in[1] : Mu->in[0];
  const CgVal *xv = &cg->v[n->in[0]], *ov = &cg->v[other];
  const int ins[2] = {n->in[0], other};
  const int grp[2] = {i, mp};
  if (numel(ov) != numel(&cg->v[so]) || numel(xv) != numel(ov) || xv->dtype != ov->dtype ||
      ov->dtype != cg->v[Mu->out].dtype || cg->v[so].dtype != xv->dtype ||
      !safe_to_defer(cg, ins, 2, i, mp, grp, 2))
    return 0;
  Mu->fused = 1;
  cg->v[so].live = 0;
  st->kind = K_SWIGLU;
  st->b = other;
  st->out = Mu->out;
  st->pos = mp;
  st->what = "swiglu";
  return 1;
}

/* rmsnorm(add(a, b)), one shape: one row pass at the norm's place; the sum
 * is stored when something besides the norm reads it (all such reads come
 * after the norm) */
static int try_add_rmsnorm(Cg *cg, int i, CgStep *st) {
  CgNode *n = &cg->n[i];
  const int h = n->out;
  int rp = -1;
  for (int u = 0; u < cg->v[h].nuses; ++u) {
    const int up = cg->v[h].uses[u];
    if (cg->n[up].op == BWPP_GOP_RMSNORM && !cg->n[up].fused && cg->n[up].in[0] == h && rp < 0) rp = up;
  }
  if (rp <= i) return 0;
  for (int u = 0; u < cg->v[h].nuses; ++u)
    if (cg->v[h].uses[u] != rp && cg->v[h].uses[u] <= rp) return 0;
  const CgNode *Rn = &cg->n[rp];
  const CgVal *av = &cg->v[n->in[0]], *bv = &cg->v[n->in[1]];
  const int gm = Rn->nin > 1 ? Rn->in[1] : -1, bt = Rn->nin > 2 ? Rn->in[2] : -1;
  const int64_t C = last_dim(&cg->v[h]);
  if (numel(av) != numel(bv) || numel(av) != numel(&cg->v[h]) || av->dtype != bv->dtype ||
      av->dtype != cg->v[h].dtype || cg->v[Rn->out].dtype != av->dtype)
    return 0;
  const int gb[2] = {gm, bt};
  for (int k = 0; k < 2; ++k)
    if (gb[k] >= 0 && (numel(&cg->v[gb[k]]) != C || cg->v[gb[k]].dtype != av->dtype)) return 0;
  const int ins[4] = {n->in[0], n->in[1], gm, bt};
  const int grp[2] = {i, rp};
  if (!safe_to_defer(cg, ins, 4, i, rp, grp, 2)) return 0;
  cg->n[rp].fused = 1;
  const int keep_h = cg->v[h].output || cg->v[h].nuses > 1;
  if (!keep_h) cg->v[h].live = 0;
  st->kind = K_ADD_RMSNORM;
  st->d = gm;
  st->e = bt;
  st->out = Rn->out;
  st->out2 = keep_h ? h : -1;
  st->pos = rp;
  st->eps = Rn->eps;
  st->what = "add_rmsnorm";
  return 1;
}

static int cmp_pos(const void *x, const void *y) {
  const CgStep *a = (const CgStep *)x, *b = (const CgStep *)y;
  return a->pos < b->pos ? -1 : a->pos > b->pos ? 1 : 0;
}

static BwppStatus lower(Cg *cg) {
  if (fuse_attention(cg) != BWPP_OK) return BWPP_ERR;
  for (int i = 0; i < cg->nn; ++i) {
    CgNode *n = &cg->n[i];
    if (n->fused) continue;
    if (is_gemm(n->op)) {
      if (lower_gemm(cg, i) != BWPP_OK) return BWPP_ERR;
      continue;
    }
    CgStep *st = new_step(cg, K_UNARY, i, n->out, op_name(n->op));
    if (!st) return cg_fail(cg, "out of memory");
    st->a = n->nin > 0 ? n->in[0] : -1;
    switch (n->op) {
      case BWPP_GOP_TRANSPOSE: st->kind = K_TRANSPOSE; break;
      case BWPP_GOP_SOFTMAX: st->kind = K_SOFTMAX; break;
      case BWPP_GOP_RMSNORM:
        st->kind = K_RMSNORM;
        st->b = n->nin > 1 ? n->in[1] : -1;
        st->c = n->nin > 2 ? n->in[2] : -1;
        st->eps = n->eps;
        break;
      case BWPP_GOP_SILU:
        st->op = 1;
        try_swiglu(cg, i, st);
        break;
      case BWPP_GOP_RESHAPE: st->op = 0; break;
      case BWPP_GOP_ADD: case BWPP_GOP_SUB: case BWPP_GOP_MUL: case BWPP_GOP_DIV:
        st->kind = K_BINARY;
        st->b = n->nin > 1 ? n->in[1] : n->in[0];
        st->op = n->op == BWPP_GOP_ADD ? 0 : n->op == BWPP_GOP_SUB ? 1 : n->op == BWPP_GOP_MUL ? 2 : 3;
        if (n->op == BWPP_GOP_ADD && n->nin == 2) try_add_rmsnorm(cg, i, st);
        break;
      case BWPP_GOP_BROADCAST:
        st->kind = K_BINARY;
        st->b = n->in[0];
        st->op = 4;
        break;
      case BWPP_GOP_SILU_GRAD: st->kind = K_SILU_GRAD; st->b = n->in[1]; break;
      case BWPP_GOP_SOFTMAX_GRAD: st->kind = K_SOFTMAX_GRAD; st->b = n->in[1]; break;
      case BWPP_GOP_RMSNORM_GRAD:
        st->kind = K_RMSNORM_GRAD;
        st->b = n->in[1];
        st->c = n->in[2];
        st->eps = n->eps;
        break;
      case BWPP_GOP_REDUCE_SUM: st->kind = K_REDUCE; break;
      case BWPP_GOP_PERMUTE:
        st->kind = K_PERMUTE;
        for (int k = 0; k < n->perm_rank; ++k) st->perm[k] = n->perm[k];
        break;
      case BWPP_GOP_REDUCE_MAX:
      case BWPP_GOP_REDUCE_MAX_MASK:
        st->kind = K_REDUCE_MAX;
        st->op = n->op == BWPP_GOP_REDUCE_MAX ? 0 : 1;
        st->axis = n->axis >= 0 ? n->axis : cg->v[n->in[0]].rank - 1;
        break;
      case BWPP_GOP_REDUCE_MAX_GRAD: /* mask * (dy broadcast to x's shape) */
        st->kind = K_BINARY;
        st->b = n->in[1];
        st->op = 2;
        st->what = "reduce_max_grad";
        break;
      default:
        return cg_fail(cg, "op %s (n%d) has no CUDA kernel", op_name(n->op), i);
    }
  }
  /* 3. launches run in node order; drop those whose results nobody reads */
  qsort(cg->s, (size_t)cg->ns, sizeof(CgStep), cmp_pos);
  char *need = (char *)calloc((size_t)cg->nv, 1), *keep = (char *)calloc((size_t)cg->ns + 1, 1);
  if (!need || !keep) {
    free(need);
    free(keep);
    return cg_fail(cg, "out of memory");
  }
  for (int i = cg->ns - 1; i >= 0; --i) {
    const CgStep *st = &cg->s[i];
    const int want2 = st->out2 >= 0 && (cg->v[st->out2].output || need[st->out2]);
    if (!cg->v[st->out].output && !need[st->out] && !want2) continue;
    keep[i] = 1;
    const int rd[6] = {st->a, st->b, st->c, st->bias, st->d, st->e};
    for (int k = 0; k < 6; ++k)
      if (rd[k] >= 0) need[rd[k]] = 1;
  }
  int w = 0;
  for (int i = 0; i < cg->ns; ++i) {
    if (keep[i]) {
      cg->s[w++] = cg->s[i];
    } else {
      cg->v[cg->s[i].out].live = 0;
      if (cg->s[i].out2 >= 0) cg->v[cg->s[i].out2].live = 0;
    }
  }
  cg->ns = w;
  free(need);
  free(keep);
  /* kernels that do not run in place get their own storage where the
   * memory plan reuses an input's buffer for the output */
  for (int i = 0; i < cg->ns; ++i) {
    const CgStep *st = &cg->s[i];
    if (st->kind != K_GEMM && st->kind != K_ATTN && st->kind != K_TRANSPOSE && st->kind != K_REDUCE &&
        st->kind != K_PERMUTE && !(st->kind == K_REDUCE_MAX && st->op == 0))
      continue;
    CgVal *o = &cg->v[st->out];
    const int rd[4] = {st->a, st->b, st->kind == K_GEMM ? -1 : st->c, st->bias};
    for (int k = 0; k < 4; ++k)
      if (rd[k] >= 0 && !cg->v[rd[k]].input && cg->v[rd[k]].buffer >= 0 &&
          cg->v[rd[k]].buffer == o->buffer)
        o->buffer = -1;
  }
  return BWPP_OK;
}

/* ---- 4. memory ---------------------------------------------------------- */

static BwppStatus layout(Cg *cg) {
  cg->buf_bytes = (size_t *)calloc((size_t)cg->nbuf + 1, sizeof(size_t));
  cg->buf_off = (size_t *)calloc((size_t)cg->nbuf + 1, sizeof(size_t));
  if (!cg->buf_bytes || !cg->buf_off) return cg_fail(cg, "out of memory");
  for (int id = 0; id < cg->nv; ++id) {
    CgVal *x = &cg->v[id];
    if (x->input || !x->live || x->producer < 0) continue;
    if (!x->known) return cg_fail(cg, "shape of v%d unknown", id);
    const size_t bytes = ((size_t)numel(x) * dt_size(x->dtype) + 255) & ~(size_t)255;
    if (x->buffer >= 0 && cg->buf_bytes[x->buffer] < bytes) cg->buf_bytes[x->buffer] = bytes;
  }
  size_t off = 0;
  for (int b = 0; b < cg->nbuf; ++b) {
    cg->buf_off[b] = off;
    off += cg->buf_bytes[b];
  }
  for (int id = 0; id < cg->nv; ++id) {
    CgVal *x = &cg->v[id];
    if (x->input || !x->live || x->producer < 0) continue;
    if (x->buffer >= 0) {
      x->offset = cg->buf_off[x->buffer];
    } else {
      x->offset = off;
      off += ((size_t)numel(x) * dt_size(x->dtype) + 255) & ~(size_t)255;
    }
  }
  cg->arena = off;
  return BWPP_OK;
}

/* ---- emission ----------------------------------------------------------- */

static void emit_meta(FILE *f, const BwppIrModule *ir) {
  /* the Metal output's bwpp.meta vocabulary, decided from the IR as
   * compiler/codegen_metal.c does, so callers gating on it keep working */
  uint32_t ops = ir ? ir->node_count : 0, regions = ir ? ir->region_count : 0;
  int has_matmul = 0, has_bias = 0, has_silu = 0, has_softmax = 0, has_rmsnorm = 0;
  for (uint32_t i = 0; ir && i < ir->node_count; ++i) {
    const BwppOpKind op = ir->nodes[i].op;
    if (op == BWPP_OP_MATMUL) has_matmul = 1;
    else if (op == BWPP_OP_ADD && (ir->nodes[i].flags & BWPP_IR_OPF_HAS_BIAS)) has_bias = 1;
    else if (op == BWPP_OP_SILU) has_silu = 1;
    else if (op == BWPP_OP_SOFTMAX) has_softmax = 1;
    else if (op == BWPP_OP_RMSNORM) has_rmsnorm = 1;
  }
  const int has_attention = ir && (ir->flags & BWPP_IRF_HAS_ATTENTION);
  fprintf(f, "// bwpp.meta: ops=%u reversible_regions=%u\n", ops, regions);
  fputs("// bwpp.meta: target=cuda\n", f);
  if (has_attention) {
    fputs("// bwpp.meta: kernel=attention_f16\n", f);
    fputs("// bwpp.meta: fused_attention_candidate=1\n", f);
  } else if (has_matmul) {
    fputs("// bwpp.meta: kernel=matmul_f16\n", f);
    if (has_bias || has_silu)
      fprintf(f, "// bwpp.meta: epilogue=%s\n",
              has_bias && has_silu ? "add_silu" : has_bias ? "add" : "silu");
  } else {
    fputs("// bwpp.meta: kernel=none\n", f);
  }
  if (has_softmax) fputs("// bwpp.meta: aux_kernel=softmax_f16\n", f);
  if (has_rmsnorm) fputs("// bwpp.meta: aux_kernel=rmsnorm_f16\n", f);
}

static void emit_shape(FILE *f, const BwppShape *s) {
  for (uint32_t i = 0; i < s->rank; ++i) fprintf(f, "%s%.*s", i ? "," : "", (int)s->dims[i].len, s->dims[i].ptr);
}

static void emit(Cg *cg, FILE *f, const BwppIrModule *ir) {
  fputs("// BW++ CUDA launch plan (bwppc --target cuda)\n", f);
  emit_meta(f, ir);
  fputs("// bwpp.dims:", f);
  for (int k = 0; k < cg->ndims; ++k) fprintf(f, " %s=%lld", cg->dim_name[k], (long long)cg->dim_val[k]);
  fputs("\n", f);
  for (int id = 0; id < cg->nv; ++id) {
    const BwppGraphValue *gv = &cg->g->values[id];
    const CgVal *x = &cg->v[id];
    fprintf(f, "// bwpp.value: v%d name=%.*s dtype=%s shape=", id, gv->name.ptr ? (int)gv->name.len : 0,
            gv->name.ptr ? gv->name.ptr : "", dt_name(x->dtype));
    emit_shape(f, &gv->shape);
    fputs(" dims=", f);
    for (int i = 0; i < x->rank; ++i) fprintf(f, "%s%lld", i ? "," : "", (long long)x->dims[i]);
    fprintf(f, " flags=%s%s", x->input ? "input" : "", x->output ? (x->input ? ",output" : "output") : "");
    if (!x->input && x->live && x->producer >= 0) {
      if (x->buffer >= 0) fprintf(f, " buffer=b%d", x->buffer);
      else fputs(" buffer=own", f);
      fprintf(f, " offset=%zu", x->offset);
    }
    fputs("\n", f);
  }
  for (int b = 0; b < cg->nbuf; ++b)
    fprintf(f, "// bwpp.buffer: b%d bytes=%zu offset=%zu\n", b, cg->buf_bytes[b], cg->buf_off[b]);
  fprintf(f, "// bwpp.arena: bytes=%zu\n", cg->arena);
  static const char *kname[] = {"gemm", "attention", "softmax", "rmsnorm", "unary", "binary",
                                "transpose", "silu_grad", "softmax_grad", "rmsnorm_grad",
                                "reduce_sum", "swiglu", "add_rmsnorm", "permute", "reduce_max"};
  static const char *bop[] = {"add", "sub", "mul", "div", "broadcast"};
  for (int i = 0; i < cg->ns; ++i) {
    const CgStep *st = &cg->s[i];
    const int rmg = st->what && strcmp(st->what, "reduce_max_grad") == 0;
    fprintf(f, "// bwpp.launch: %d %s node=n%d", i, rmg ? "reduce_max_grad" : kname[st->kind], st->pos);
    switch (rmg ? -1 : st->kind) {
      case -1: fprintf(f, " mask=v%d dy=v%d", st->a, st->b); break;
      case K_PERMUTE:
        fprintf(f, " x=v%d perm=", st->a);
        for (int k = 0; k < cg->v[st->a].rank; ++k) fprintf(f, "%s%d", k ? "," : "", st->perm[k]);
        break;
      case K_REDUCE_MAX:
        fprintf(f, " x=v%d axis=%d mode=%s", st->a, st->axis, st->op ? "mask" : "values");
        break;
      case K_GEMM:
        fprintf(f, " a=v%d b=v%d", st->a, st->b);
        if (st->a_t) fputs(" a_t=1", f);
        if (st->b_t) fputs(" b_t=1", f);
        if (st->bias >= 0) fprintf(f, " bias=v%d", st->bias);
        if (st->silu) fputs(" silu=1", f);
        if (st->c >= 0) fprintf(f, " %s=v%d", st->res_mul ? "gate" : "residual", st->c);
        break;
      case K_ATTN:
        fprintf(f, " q=v%d k=v%d v=v%d scale=1 causal=0", st->a, st->b, st->c);
        break;
      case K_RMSNORM:
        fprintf(f, " x=v%d", st->a);
        if (st->b >= 0) fprintf(f, " gamma=v%d", st->b);
        if (st->c >= 0) fprintf(f, " beta=v%d", st->c);
        fprintf(f, " eps=%.9g", st->eps);
        break;
      case K_ADD_RMSNORM:
        fprintf(f, " a=v%d b=v%d", st->a, st->b);
        if (st->d >= 0) fprintf(f, " gamma=v%d", st->d);
        if (st->e >= 0) fprintf(f, " beta=v%d", st->e);
        if (st->out2 >= 0) fprintf(f, " sum=v%d", st->out2);
        fprintf(f, " eps=%.9g", st->eps);
        break;
      case K_SWIGLU: fprintf(f, " x=v%d y=v%d", st->a, st->b); break;
      case K_UNARY: fprintf(f, " op=%s x=v%d", st->op == 1 ? "silu" : "copy", st->a); break;
      case K_BINARY: fprintf(f, " op=%s a=v%d b=v%d", bop[st->op], st->a, st->b); break;
      case K_SILU_GRAD: fprintf(f, " x=v%d dy=v%d", st->a, st->b); break;
      case K_SOFTMAX_GRAD: fprintf(f, " y=v%d dy=v%d", st->a, st->b); break;
      case K_RMSNORM_GRAD:
        fprintf(f, " x=v%d gamma=v%d dy=v%d eps=%.9g", st->a, st->b, st->c, st->eps);
        break;
      default: fprintf(f, " x=v%d", st->a); break;
    }
    fprintf(f, " out=v%d\n", st->out);
  }
}

static void cg_free(Cg *cg) {
  for (int i = 0; i < cg->nv; ++i) free(cg->v[i].uses);
  free(cg->v);
  free(cg->n);
  free(cg->s);
  free(cg->buf_bytes);
  free(cg->buf_off);
}

BwppStatus bwpp_codegen_cuda(const BwppIrModule *ir, const BwppGraph *graph, const char *dims,
                             const char *out_path) {
  if (!graph || !out_path) return BWPP_ERR;
  Cg cg;
  memset(&cg, 0, sizeof(cg));
  cg.g = graph;
  BwppStatus rc = parse_dims(&cg, dims);
  BwppMemPlan *mp = NULL;
  if (rc == BWPP_OK) {
    cg.nv = (int)graph->value_count;
    cg.nn = (int)graph->node_count;
    cg.v = (CgVal *)calloc((size_t)cg.nv + 1, sizeof(CgVal));
    cg.n = (CgNode *)calloc((size_t)cg.nn + 1, sizeof(CgNode));
    mp = bwpp_mem_plan_build(graph);
    if (!cg.v || !cg.n || !mp) rc = cg_fail(&cg, "out of memory");
  }
  for (int id = 0; rc == BWPP_OK && id < cg.nv; ++id) {
    const BwppGraphValue *gv = &graph->values[id];
    CgVal *x = &cg.v[id];
    if (gv->id != (uint32_t)id) {
      rc = cg_fail(&cg, "value %d has id %u", id, gv->id);
      break;
    }
    x->dtype = gv->dtype == BWPP_DTYPE_F16 ? DT_F16 : gv->dtype == BWPP_DTYPE_BF16 ? DT_BF16
             : gv->dtype == BWPP_DTYPE_F32 ? DT_F32 : -1;
    if (x->dtype < 0) rc = cg_fail(&cg, "v%d: dtype not f16 / bf16 / f32", id);
    x->input = (gv->flags & BWPP_GRAPH_VALUE_INPUT) != 0;
    x->output = !x->input && (gv->flags & BWPP_GRAPH_VALUE_OUTPUT) != 0;
    x->producer = -1;
    x->live = 1;
    x->buffer = (!x->input && mp->value_to_buffer[id] != UINT32_MAX) ? (int)mp->value_to_buffer[id] : -1;
    if (rc == BWPP_OK) rc = resolve(&cg, id);
  }
  if (mp) cg.nbuf = (int)mp->buffer_count;
  for (int i = 0; rc == BWPP_OK && i < cg.nn; ++i) {
    const BwppGraphNode *gn = &graph->nodes[i];
    CgNode *n = &cg.n[i];
    n->op = gn->op;
    n->nin = (int)gn->input_count;
    n->out = (int)gn->output;
    n->eps = gn->attr.has_epsilon ? gn->attr.epsilon : 1e-5f;
    n->axis = gn->attr.has_axis ? gn->attr.axis : -1;
    n->perm_rank = (int)gn->attr.perm_rank;
    for (int k = 0; k < n->perm_rank && k < BWPP_GRAPH_MAX_DIMS; ++k) n->perm[k] = (int)gn->attr.perm[k];
    if (n->out < 0 || n->out >= cg.nv || cg.v[n->out].producer >= 0) {
      rc = cg_fail(&cg, "node n%d: bad or repeated output", i);
      break;
    }
    cg.v[n->out].producer = i;
    for (int k = 0; k < n->nin; ++k) {
      n->in[k] = (int)gn->inputs[k];
      if (n->in[k] < 0 || n->in[k] >= cg.nv) {
        rc = cg_fail(&cg, "node n%d reads unknown v%d", i, n->in[k]);
        break;
      }
      const CgVal *src = &cg.v[n->in[k]];
      if (!src->input && (src->producer < 0 || src->producer >= i)) {
        rc = cg_fail(&cg, "nodes are not in dependency order at n%d", i);
        break;
      }
      if (!add_use(&cg.v[n->in[k]], i)) rc = cg_fail(&cg, "out of memory");
    }
  }
  for (int i = 0; rc == BWPP_OK && i < cg.nn; ++i) rc = infer(&cg, i);
  if (rc == BWPP_OK) rc = lower(&cg);
  if (rc == BWPP_OK) rc = layout(&cg);
  if (rc == BWPP_OK) {
    FILE *f = fopen(out_path, "w");
    if (!f) {
      rc = cg_fail(&cg, "cannot open %s", out_path);
    } else {
      emit(&cg, f, ir);
      if (fclose(f) != 0) rc = cg_fail(&cg, "cannot write %s", out_path);
    }
  }
  if (rc != BWPP_OK) fprintf(stderr, "codegen cuda: %s\n", cg.err);
  if (mp) bwpp_mem_plan_destroy(mp);
  cg_free(&cg);
  return rc;
}
