#ifndef BWPP_CODEGEN_CUDA_H
#define BWPP_CODEGEN_CUDA_H

/* `bwppc --target cuda`: the launch plan for the B200 runtime
 * (runtime/cuda), emitted in place of compiler/codegen_metal.c's Metal
 * source (compiler/main.c:186 calls bwpp_codegen_metal; the patch in this
 * directory calls this function instead when --target cuda is given).
 *
 * The plan is text.  It keeps the `// bwpp.meta:` lines of the Metal output
 * (kernel=, epilogue=, aux_kernel=, derived from the IR as
 * compiler/codegen_metal.c:17-123 and 273-356 derive them), so callers that
 * gate on those tags keep working, and adds:
 *   // bwpp.dims:   the symbolic dims bound by --dims (shapes are static)
 *   // bwpp.value:  every graph value: id, name, dtype, symbolic and bound
 *                   shape, input / output flags, and for a value the plan
 *                   materialises its byte offset in the arena
 *   // bwpp.buffer: the memory plan's buffers (compiler/mem_plan.c:43-146)
 *                   with byte sizes from the bound dims and arena offsets
 *   // bwpp.arena:  total bytes (one cudaMalloc per GPU)
 *   // bwpp.launch: one line per kernel launch, in order: the kernel, its
 *                   operand value ids and its fused epilogue
 * The fusion decisions are made here, on the graph: attention
 * (compiler/graph_ir.c:1852-1899 pattern), transposes folded into GEMM
 * operand layouts, bias found by dataflow (also behind a reshape, which
 * compiler/graph_ir.c:760-767 misses), SiLU, the SwiGLU gate and residual
 * adds in the GEMM epilogue, swiglu and residual + norm as single kernels
 * (spec/llm-primitives.md:17-22). */

#include "bwpp.h"
#include "graph_ir.h"
#include "ir.h"

/* dims: "NAME=VALUE,..." binding every symbolic dim of the graph. */
BwppStatus bwpp_codegen_cuda(const BwppIrModule *ir, const BwppGraph *graph,
                             const char *dims, const char *out_path);

#endif
