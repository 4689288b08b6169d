/*
 * bwpp_bench_cuda -- the reference's CPU bench (bench/bench_cpu.c:37-169)
 * with a --cuda mode, written against the B200 runtime's C ABI only.
 *
 * Same command line (--iters --m --n --k --rows --cols --json --metal) and the
 * same JSON keys (matmul.{M,N,K,iters,time_s,gflops}, softmax / rmsnorm
 * .{rows,cols,iters,time_s}) as bench/bench_cpu.c:45-63,142-158, so
 * bench/bench_regress.py reads its output unchanged.  Inputs use the bench's
 * ramp fill (i*cols + j + 1) * scale (bench_cpu.c:14-20, 82-83).
 *
 *   --cuda        run on the GPU: buffers from one arena (bwpp_cuda_arena_*),
 *                 timed calls of the CPU-signature mirrors bwpp_cuda_*_f32 on
 *                 device-resident data (each call is synchronous)
 *   --device N    GPU ordinal (default 0)
 * Without --cuda the same loop runs bwpp_cuda_*_f32 on HOST buffers, which
 * stages every call through the device (host <-> device copies timed).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "bwpp_cuda.h"

/* monotonic wall clock in seconds, for the timed loops */
static double wall_seconds(void) {
  struct timespec t;
  if (clock_gettime(CLOCK_MONOTONIC, &t) != 0) return 0.0;
  return 1e-9 * (double)t.tv_nsec + (double)t.tv_sec;
}

static void ramp(float *dst, uint32_t rows, uint32_t cols, float scale) {
  for (uint32_t i = 0; i < rows; ++i)
    for (uint32_t j = 0; j < cols; ++j) dst[(size_t)i * cols + j] = (float)(i * cols + j + 1) * scale;
}

/* Echoes the compiler output's tag lines (bwpp.meta / bwpp.plan / bwpp.launch)
 * so a run records which kernels and epilogue the compiler chose. */
static void echo_tags(const char *path) {
  static const char *const tags[] = {"bwpp.meta:", "bwpp.plan:", "bwpp.launch:"};
  FILE *src = fopen(path, "r");
  if (src == NULL) {
    fprintf(stderr, "bench: cannot open compiler output %s\n", path);
    return;
  }
  char buf[1024];
  while (fgets(buf, (int)sizeof(buf), src) != NULL) {
    for (size_t t = 0; t < sizeof(tags) / sizeof(tags[0]); ++t) {
      if (strstr(buf, tags[t]) != NULL) {
        fputs(buf, stdout);
        break;
      }
    }
  }
  fclose(src);
}

int main(int argc, char **argv) {
  uint32_t M = 256, N = 256, K = 256, iters = 10, rows = 256, cols = 256;
  const char *metal_path = NULL, *json_path = NULL;
  int use_cuda = 0, device = 0;
  for (int i = 1; i < argc; ++i) {
    if (!strcmp(argv[i], "--iters") && i + 1 < argc) iters = (uint32_t)strtoul(argv[++i], NULL, 10);
    else if (!strcmp(argv[i], "--m") && i + 1 < argc) M = (uint32_t)strtoul(argv[++i], NULL, 10);
    else if (!strcmp(argv[i], "--n") && i + 1 < argc) N = (uint32_t)strtoul(argv[++i], NULL, 10);
    else if (!strcmp(argv[i], "--k") && i + 1 < argc) K = (uint32_t)strtoul(argv[++i], NULL, 10);
    else if (!strcmp(argv[i], "--rows") && i + 1 < argc) rows = (uint32_t)strtoul(argv[++i], NULL, 10);
    else if (!strcmp(argv[i], "--cols") && i + 1 < argc) cols = (uint32_t)strtoul(argv[++i], NULL, 10);
    else if (!strcmp(argv[i], "--metal") && i + 1 < argc) metal_path = argv[++i];
    else if (!strcmp(argv[i], "--json") && i + 1 < argc) json_path = argv[++i];
    else if (!strcmp(argv[i], "--cuda")) use_cuda = 1;
    else if (!strcmp(argv[i], "--device") && i + 1 < argc) device = atoi(argv[++i]);
  }
  if (metal_path) {
    printf("== MSL metadata ==\n");
    echo_tags(metal_path);
  }
  const size_t na = (size_t)M * K, nb = (size_t)K * N, nc = (size_t)M * N, nx = (size_t)rows * cols;
  float *a = malloc(na * 4), *b = malloc(nb * 4), *c = malloc(nc * 4), *bias = calloc(N, 4);
  float *x = malloc(nx * 4), *y = malloc(nx * 4), *gamma = malloc((size_t)cols * 4);
  if (!a || !b || !c || !bias || !x || !y || !gamma) {
    fprintf(stderr, "bench: alloc failed\n");
    return 1;
  }
  ramp(a, M, K, 0.01f);
  ramp(b, K, N, 0.02f);
  ramp(x, rows, cols, 0.01f);
  for (uint32_t i = 0; i < cols; ++i) gamma[i] = 1.0f;

  /* buffers the timed calls use: host arrays, or arena copies on the GPU */
  float *ta = a, *tb = b, *tc = c, *tbias = bias, *tx = x, *ty = y, *tg = gamma;
  BwppCudaArena arena;
  BwppCudaCtx *ctx = NULL;
  if (use_cuda) {
    const size_t bytes = (na + nb + nc + N + 2 * nx + cols) * 4 + 16 * 256;
    if (!bwpp_cuda_arena_init(&arena, bytes, device) ||
        bwpp_cuda_ctx_create(&ctx, device, NULL) != BWPP_CUDA_OK) {
      fprintf(stderr, "bench: no CUDA device %d\n", device);
      return 1;
    }
    ta = bwpp_cuda_arena_alloc(&arena, na * 4, 256);
    tb = bwpp_cuda_arena_alloc(&arena, nb * 4, 256);
    tc = bwpp_cuda_arena_alloc(&arena, nc * 4, 256);
    tbias = bwpp_cuda_arena_alloc(&arena, (size_t)N * 4, 256);
    tx = bwpp_cuda_arena_alloc(&arena, nx * 4, 256);
    ty = bwpp_cuda_arena_alloc(&arena, nx * 4, 256);
    tg = bwpp_cuda_arena_alloc(&arena, (size_t)cols * 4, 256);
    if (bwpp_cuda_copy(ctx, ta, a, na * 4) || bwpp_cuda_copy(ctx, tb, b, nb * 4) ||
        bwpp_cuda_copy(ctx, tbias, bias, (size_t)N * 4) || bwpp_cuda_copy(ctx, tx, x, nx * 4) ||
        bwpp_cuda_copy(ctx, tg, gamma, (size_t)cols * 4)) {
      fprintf(stderr, "bench: upload failed: %s\n", bwpp_cuda_ctx_last_error(ctx));
      return 1;
    }
  }
  /* one untimed call of each op (kernel set-up, scratch) */
  bwpp_cuda_matmul_f32(ta, tb, tc, M, N, K, K, N, N, tbias, 0, 0);
  bwpp_cuda_softmax_f32(tx, ty, rows, cols, cols);
  bwpp_cuda_rmsnorm_f32(tx, ty, tg, NULL, rows, cols, cols, 1e-5f);
  if (bwpp_cuda_last_status() != BWPP_CUDA_OK) {
    fprintf(stderr, "bench: warm-up failed: %s\n", bwpp_cuda_status_string(bwpp_cuda_last_status()));
    return 1;
  }

  double t0 = wall_seconds();
  for (uint32_t i = 0; i < iters; ++i) bwpp_cuda_matmul_f32(ta, tb, tc, M, N, K, K, N, N, tbias, 0, 0);
  double t1 = wall_seconds();
  const double matmul_secs = t1 - t0;
  const double gflops = 2.0 * M * N * K * iters / 1e9 / (matmul_secs > 0 ? matmul_secs : 1.0);
  printf("matmul: M=%u N=%u K=%u iters=%u time=%.6fs gflops=%.2f%s\n", M, N, K, iters, matmul_secs,
         gflops, use_cuda ? " (cuda)" : " (cuda, host buffers)");
  t0 = wall_seconds();
  for (uint32_t i = 0; i < iters; ++i) bwpp_cuda_softmax_f32(tx, ty, rows, cols, cols);
  t1 = wall_seconds();
  const double softmax_secs = t1 - t0;
  printf("softmax: rows=%u cols=%u iters=%u time=%.6fs\n", rows, cols, iters, softmax_secs);
  t0 = wall_seconds();
  for (uint32_t i = 0; i < iters; ++i) bwpp_cuda_rmsnorm_f32(tx, ty, tg, NULL, rows, cols, cols, 1e-5f);
  t1 = wall_seconds();
  const double rmsnorm_secs = t1 - t0;
  printf("rmsnorm: rows=%u cols=%u iters=%u time=%.6fs\n", rows, cols, iters, rmsnorm_secs);
  const int status = bwpp_cuda_last_status();

  if (json_path) {
    FILE *jf = fopen(json_path, "w");
    if (!jf) {
      fprintf(stderr, "bench: failed to write json %s\n", json_path);
    } else {
      fprintf(jf,
              "{\n"
              "  \"matmul\": {\"M\": %u, \"N\": %u, \"K\": %u, \"iters\": %u, \"time_s\": %.9f, \"gflops\": %.3f},\n"
              "  \"softmax\": {\"rows\": %u, \"cols\": %u, \"iters\": %u, \"time_s\": %.9f},\n"
              "  \"rmsnorm\": {\"rows\": %u, \"cols\": %u, \"iters\": %u, \"time_s\": %.9f},\n"
              "  \"backend\": \"%s\"\n"
              "}\n",
              M, N, K, iters, matmul_secs, gflops, rows, cols, iters, softmax_secs, rows, cols, iters,
              rmsnorm_secs, use_cuda ? "cuda" : "cuda-host-buffers");
      fclose(jf);
    }
  }
  if (use_cuda) {
    bwpp_cuda_ctx_destroy(ctx);
    bwpp_cuda_arena_destroy(&arena);
  }
  free(a); free(b); free(c); free(bias); free(x); free(y); free(gamma);
  return status == BWPP_CUDA_OK ? 0 : 1;
}
