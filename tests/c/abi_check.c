/* abi_check.c -- the C ABI exercised from C, as a C or Swift host binds it.
 *
 * Compiled with gcc against include/tgsample.h only (no C++ and no torch) and
 * linked to libtgsample.so and the CUDA runtime.  Checks the struct layouts the
 * header fixes, then samples the committed fixture (tests/golden/c_abi_case.bin,
 * expected ids and probabilities from the CPU oracle) through tg_sample with
 * device buffers and through tg_sample_host with host buffers, and compares
 * both bit for bit.  Exit status 0 on success.
 *
 * Usage: abi_check <c_abi_case.bin> [device]
 */
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "tgsample.h"

_Static_assert(sizeof(tg_row_params) == 32, "tg_row_params is 32 bytes");
_Static_assert(offsetof(tg_row_params, top_k) == 24, "tg_row_params.top_k at byte 24");
_Static_assert(sizeof(tg_shard_cand) == 8, "tg_shard_cand is 8 bytes");
_Static_assert(sizeof(tg_shard_record) == 16 + 8 * TG_SHARD_CAP, "tg_shard_record layout");
_Static_assert(offsetof(tg_shard_record, cand) == 16, "tg_shard_record.cand at byte 16");

static int fail(const char* what) {
  fprintf(stderr, "abi_check: %s\n", what);
  return 1;
}

#define CK(call)                                                              \
  do {                                                                        \
    int32_t rc_ = (call);                                                     \
    if (rc_ != TG_OK) {                                                       \
      fprintf(stderr, "abi_check: %s -> %d (%s)\n", #call, rc_, tg_last_error_string()); \
      return 1;                                                               \
    }                                                                         \
  } while (0)

#define CU(call)                                                              \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess) {                                                  \
      fprintf(stderr, "abi_check: %s -> %s\n", #call, cudaGetErrorString(e_)); \
      return 1;                                                               \
    }                                                                         \
  } while (0)

static void* dev_copy(const void* h, size_t n) {
  void* d = NULL;
  if (cudaMalloc(&d, n) != cudaSuccess) return NULL;
  if (cudaMemcpy(d, h, n, cudaMemcpyHostToDevice) != cudaSuccess) return NULL;
  return d;
}

int main(int argc, char** argv) {
  if (argc < 2) return fail("usage: abi_check <c_abi_case.bin> [device]");
  const int device = argc > 2 ? atoi(argv[2]) : 0;
  FILE* f = fopen(argv[1], "rb");
  if (!f) return fail("cannot open the fixture");
  int32_t hdr[4];
  if (fread(hdr, 4, 4, f) != 4) return fail("short header");
  const int32_t dtype = hdr[0], V = hdr[1], B = hdr[2], HS = hdr[3];
  const size_t esz = dtype == TG_DTYPE_BF16 ? 2 : 4;
  const size_t nlog = (size_t)B * V * esz;
  unsigned char* logits = malloc(nlog);
  tg_row_params* params = malloc(sizeof(tg_row_params) * B);
  int32_t* hist = malloc(sizeof(int32_t) * B * HS);
  int32_t* hlen = malloc(sizeof(int32_t) * B);
  float* u = malloc(sizeof(float) * B);
  int32_t* want = malloc(sizeof(int32_t) * B);
  float* want_p = malloc(sizeof(float) * B);
  int32_t* got = malloc(sizeof(int32_t) * B);
  float* got_p = malloc(sizeof(float) * B);
  if (fread(logits, 1, nlog, f) != nlog || fread(params, sizeof(tg_row_params), B, f) != (size_t)B ||
      fread(hist, 4, (size_t)B * HS, f) != (size_t)B * HS || fread(hlen, 4, B, f) != (size_t)B ||
      fread(u, 4, B, f) != (size_t)B || fread(want, 4, B, f) != (size_t)B || fread(want_p, 4, B, f) != (size_t)B)
    return fail("short fixture");
  fclose(f);

  tg_sampler* s = NULL;
  CK(tg_sampler_create(device, V, B, &s));
  CU(cudaSetDevice(device));

  /* device entry point */
  void* d_logits = dev_copy(logits, nlog);
  void* d_params = dev_copy(params, sizeof(tg_row_params) * B);
  void* d_hist = dev_copy(hist, sizeof(int32_t) * B * HS);
  void* d_hlen = dev_copy(hlen, sizeof(int32_t) * B);
  void* d_u = dev_copy(u, sizeof(float) * B);
  void *d_out = NULL, *d_prob = NULL;
  CU(cudaMalloc(&d_out, sizeof(int32_t) * B));
  CU(cudaMalloc(&d_prob, sizeof(float) * B));
  if (!d_logits || !d_params || !d_hist || !d_hlen || !d_u) return fail("device copies failed");
  CK(tg_sample(s, d_logits, dtype, V, B, (const tg_row_params*)d_params, (const int32_t*)d_hist,
               (const int32_t*)d_hlen, HS, NULL, 0, NULL, (const float*)d_u, (int32_t*)d_out,
               (float*)d_prob, NULL));
  CU(cudaDeviceSynchronize());
  CU(cudaMemcpy(got, d_out, sizeof(int32_t) * B, cudaMemcpyDeviceToHost));
  CU(cudaMemcpy(got_p, d_prob, sizeof(float) * B, cudaMemcpyDeviceToHost));
  for (int b = 0; b < B; b++) {
    if (got[b] != want[b] || memcmp(&got_p[b], &want_p[b], 4) != 0) {
      fprintf(stderr, "abi_check: tg_sample row %d: id %d prob %.9g, expected %d %.9g\n", b, got[b],
              got_p[b], want[b], want_p[b]);
      return 1;
    }
  }

  /* host entry point */
  memset(got, 0xff, sizeof(int32_t) * B);
  CK(tg_sample_host(s, logits, dtype, V, B, params, hist, hlen, HS, NULL, 0, NULL, u, got, got_p));
  for (int b = 0; b < B; b++) {
    if (got[b] != want[b] || memcmp(&got_p[b], &want_p[b], 4) != 0) {
      fprintf(stderr, "abi_check: tg_sample_host row %d: id %d, expected %d\n", b, got[b], want[b]);
      return 1;
    }
  }

  /* errors come back as status codes, with a message */
  if (tg_sample(s, d_logits, 7, V, B, (const tg_row_params*)d_params, NULL, NULL, 0, NULL, 0, NULL,
                (const float*)d_u, (int32_t*)d_out, NULL, NULL) != TG_ERR_INVALID_ARG)
    return fail("a bad dtype was accepted");
  if (strlen(tg_last_error_string()) == 0) return fail("no error message");

  CK(tg_sampler_destroy(s));
  cudaFree(d_logits); cudaFree(d_params); cudaFree(d_hist); cudaFree(d_hlen); cudaFree(d_u);
  cudaFree(d_out); cudaFree(d_prob);
  printf("abi_check: %d rows equal through tg_sample and tg_sample_host\n", B);
  return 0;
}
