/* A host program in plain C that drives the mixer through the C ABI alone (no Python, no
 * PyTorch): forward and backward of one SPARC layer, float32, inputs from closed-form patterns.
 * Writes y, dx and the parameter gradients to the binary file named by argv[1]
 * (tests/test_gpu_c_abi.py rebuilds the same inputs and checks them against the oracle). */
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "sparc_b200.h"

#define B 2
#define T 37
#define W 10
#define M (W / 2)

static float* dev(const float* h, size_t n) {
  float* d = NULL;
  if (cudaMalloc((void**)&d, n * sizeof(float)) != cudaSuccess) exit(2);
  if (h) cudaMemcpy(d, h, n * sizeof(float), cudaMemcpyHostToDevice);
  else cudaMemset(d, 0, n * sizeof(float));
  return d;
}

static void put(FILE* f, const float* d, size_t n) {
  float* h = (float*)malloc(n * sizeof(float));
  cudaMemcpy(h, d, n * sizeof(float), cudaMemcpyDeviceToHost);
  fwrite(h, sizeof(float), n, f);
  free(h);
}

int main(int argc, char** argv) {
  if (argc < 2) return 1;
  float x[B * T * W], dy[B * T * W];
  float nu_log[M], theta_log[M], wlg[M], wpr[M], wrr[M], pd[W + 1], rd[W + 1];
  for (int i = 0; i < B * T * W; ++i) {
    x[i] = sinf(0.37f * (float)i) * 1.3f;
    dy[i] = cosf(0.21f * (float)i + 0.5f);
  }
  for (int m = 0; m < M; ++m) {
    nu_log[m] = -3.0f + 0.4f * (float)m;
    theta_log[m] = -1.0f + 0.3f * (float)m;
    wlg[m] = -0.5f - 0.1f * (float)m;
    wpr[m] = 0.3f * sinf((float)m);
    wrr[m] = 0.2f * cosf((float)m);
  }
  for (int j = 0; j <= W; ++j) {
    pd[j] = 0.15f * sinf(1.7f * (float)j);
    rd[j] = 0.15f * cosf(1.3f * (float)j);
  }
  const int chunks = (int)sparc_mixer_carry_chunks(T, SPARC_DTYPE_F32);
  const int cf = sparc_mixer_controls_floats();
  float *d_x = dev(x, B * T * W), *d_dy = dev(dy, B * T * W), *d_y = dev(NULL, B * T * W), *d_dx = dev(NULL, B * T * W);
  float *d_nu = dev(nu_log, M), *d_th = dev(theta_log, M), *d_wlg = dev(wlg, M), *d_wpr = dev(wpr, M),
        *d_wrr = dev(wrr, M), *d_pd = dev(pd, W + 1), *d_rd = dev(rd, W + 1);
  float* d_carry = dev(NULL, (size_t)B * chunks * M * 2);
  float* d_ctl = dev(NULL, (size_t)B * T * cf);
  float* g[8];
  const size_t gn[8] = {M, M, W + 1, W + 1, M, M, M, M};
  for (int i = 0; i < 8; ++i) g[i] = dev(NULL, gn[i]);
  const size_t wsb = sparc_mixer_workspace_bytes(B, T, W, SPARC_DTYPE_F32);
  void* ws = NULL;
  if (wsb == 0 || cudaMalloc(&ws, wsb) != cudaSuccess) return 3;
  cudaMemset(ws, 0, wsb);

  SparcMixerFwdArgs fa;
  memset(&fa, 0, sizeof(fa));
  fa.x = d_x; fa.y = d_y;
  fa.nu_log = d_nu; fa.theta_log = d_th; fa.phase_direction = d_pd; fa.radial_direction = d_rd;
  fa.write_log_gain = d_wlg; fa.write_phase_response = d_wpr; fa.write_radial_response = d_wrr;
  fa.carry = d_carry; fa.controls = d_ctl;
  fa.workspace = ws; fa.workspace_bytes = wsb;
  fa.batch = B; fa.length = T; fa.width = W; fa.dtype = SPARC_DTYPE_F32;
  int rc = sparc_mixer_forward(&fa, NULL);
  if (rc != SPARC_OK) { fprintf(stderr, "forward: %d %s\n", rc, sparc_last_error()); return 4; }

  SparcMixerBwdArgs ba;
  memset(&ba, 0, sizeof(ba));
  ba.x = d_x; ba.y = d_y; ba.dy = d_dy; ba.dx = d_dx;
  ba.nu_log = d_nu; ba.theta_log = d_th; ba.phase_direction = d_pd; ba.radial_direction = d_rd;
  ba.write_log_gain = d_wlg; ba.write_phase_response = d_wpr; ba.write_radial_response = d_wrr;
  ba.carry = d_carry; ba.controls = d_ctl;
  ba.grad_nu_log = g[0]; ba.grad_theta_log = g[1]; ba.grad_phase_direction = g[2]; ba.grad_radial_direction = g[3];
  ba.grad_write_log_gain = g[4]; ba.grad_energy_response = g[5]; ba.grad_write_phase_response = g[6];
  ba.grad_write_radial_response = g[7];
  ba.workspace = ws; ba.workspace_bytes = wsb;
  ba.batch = B; ba.length = T; ba.width = W; ba.dtype = SPARC_DTYPE_F32;
  rc = sparc_mixer_backward(&ba, NULL);
  if (rc != SPARC_OK) { fprintf(stderr, "backward: %d %s\n", rc, sparc_last_error()); return 5; }
  if (cudaDeviceSynchronize() != cudaSuccess) return 6;

  FILE* f = fopen(argv[1], "wb");
  if (!f) return 7;
  put(f, d_y, B * T * W);
  put(f, d_dx, B * T * W);
  for (int i = 0; i < 8; ++i) put(f, g[i], gn[i]);
  fclose(f);
  printf("ok\n");
  return 0;
}
