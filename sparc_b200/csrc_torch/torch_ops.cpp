// TORCH_LIBRARY registration of the libsparc_b200 C ABI: the mixer forward / backward, the
// decode step and the real-mode scans as PyTorch operators (torch.ops.sparc_b200.*) on CUDA
// tensors, enqueued on PyTorch's current stream. Each operator allocates its outputs and a
// zeroed workspace from PyTorch's caching allocator and calls the C entry point; errors become
// exceptions with the library's message. No arithmetic here: the kernels are in libsparc_b200.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <optional>
#include <tuple>

#include "sparc_b200.h"

namespace {

void check(int rc, const char* what) {
  TORCH_CHECK(rc == SPARC_OK, what, " failed (", rc, "): ", sparc_last_error());
}

int dtype_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kFloat) return SPARC_DTYPE_F32;
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, "sparc_b200: float32 or bfloat16 activations");
  return SPARC_DTYPE_BF16;
}

at::Tensor f32(const at::Tensor& t) { return t.to(at::kFloat).contiguous(); }

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

at::Tensor workspace(const at::Tensor& like, size_t bytes) {
  return at::zeros({(int64_t)bytes}, like.options().dtype(at::kByte));
}

// SPARCMixer forward (sparc-kernal/forward/scan.py:1398-1603): (y, last_r, last_i, carry, controls,
// states).
std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> mixer_forward(
    const at::Tensor& x_in, const at::Tensor& nu_log, const at::Tensor& theta_log, const at::Tensor& phase_direction,
    const at::Tensor& radial_direction, const at::Tensor& write_log_gain, const at::Tensor& write_phase_response,
    const at::Tensor& write_radial_response) {
  TORCH_CHECK(x_in.is_cuda() && x_in.dim() == 3, "mixer_forward: x must be a CUDA [batch, length, width] tensor");
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor x = x_in.contiguous();
  const int64_t B = x.size(0), T = x.size(1), W = x.size(2), M = W / 2;
  const int dt = dtype_code(x);
  const at::Tensor p[7] = {f32(nu_log), f32(theta_log), f32(phase_direction), f32(radial_direction),
                           f32(write_log_gain), f32(write_phase_response), f32(write_radial_response)};
  at::Tensor y = at::empty_like(x);
  at::Tensor states = at::empty_like(x);  // every token's state, for mixer_backward
  auto fo = x.options().dtype(at::kFloat);
  at::Tensor last_r = at::empty({B, M}, fo), last_i = at::empty({B, M}, fo);
  at::Tensor carry = at::empty({B, sparc_mixer_carry_chunks(T, dt), M, 2}, fo);
  at::Tensor controls = at::empty({B, T, sparc_mixer_controls_floats()}, fo);
  const size_t wsb = sparc_mixer_workspace_bytes(B, T, (int)W, dt);
  TORCH_CHECK(wsb > 0, "mixer_forward: unsupported shape (", sparc_last_error(), ")");
  at::Tensor ws = workspace(x, wsb);
  SparcMixerFwdArgs a = {};
  a.x = x.data_ptr();
  a.y = y.data_ptr();
  a.nu_log = p[0].data_ptr<float>();
  a.theta_log = p[1].data_ptr<float>();
  a.phase_direction = p[2].data_ptr<float>();
  a.radial_direction = p[3].data_ptr<float>();
  a.write_log_gain = p[4].data_ptr<float>();
  a.write_phase_response = p[5].data_ptr<float>();
  a.write_radial_response = p[6].data_ptr<float>();
  a.last_r = last_r.data_ptr<float>();
  a.last_i = last_i.data_ptr<float>();
  a.carry = carry.data_ptr<float>();
  a.controls = controls.data_ptr<float>();
  a.workspace = ws.data_ptr();
  a.workspace_bytes = wsb;
  a.batch = B;
  a.length = T;
  a.width = (int)W;
  a.dtype = dt;
  a.states = states.data_ptr();
  check(sparc_mixer_forward(&a, stream_of(x)), "sparc_mixer_forward");
  return {y, last_r, last_i, carry, controls, states};
}

// Its backward: (dx, grad of each of the eight parameters in the module's order). With the
// forward's states (its sixth output) the gradient kernel reads them instead of replaying them.
std::vector<at::Tensor> mixer_backward(const at::Tensor& x_in, const at::Tensor& y, const at::Tensor& dy_in,
                                       const at::Tensor& nu_log, const at::Tensor& theta_log,
                                       const at::Tensor& phase_direction, const at::Tensor& radial_direction,
                                       const at::Tensor& write_log_gain, const at::Tensor& write_phase_response,
                                       const at::Tensor& write_radial_response, const at::Tensor& carry,
                                       const at::Tensor& controls, const std::optional<at::Tensor>& states) {
  TORCH_CHECK(x_in.is_cuda() && x_in.dim() == 3 && y.sizes() == x_in.sizes() && dy_in.sizes() == x_in.sizes(),
              "mixer_backward: x, y and dy must be CUDA [batch, length, width] tensors of one shape");
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor x = x_in.contiguous(), dy = dy_in.to(x.scalar_type()).contiguous(), yc = y.contiguous();
  const int64_t B = x.size(0), T = x.size(1), W = x.size(2), M = W / 2;
  const int dt = dtype_code(x);
  const at::Tensor p[7] = {f32(nu_log), f32(theta_log), f32(phase_direction), f32(radial_direction),
                           f32(write_log_gain), f32(write_phase_response), f32(write_radial_response)};
  auto fo = x.options().dtype(at::kFloat);
  at::Tensor dx = at::empty_like(x);
  std::vector<at::Tensor> g = {at::empty({M}, fo), at::empty({M}, fo), at::empty({W + 1}, fo), at::empty({W + 1}, fo),
                               at::empty({M}, fo), at::empty({M}, fo), at::empty({M}, fo), at::empty({M}, fo)};
  const size_t wsb = sparc_mixer_workspace_bytes(B, T, (int)W, dt);
  TORCH_CHECK(wsb > 0, "mixer_backward: unsupported shape (", sparc_last_error(), ")");
  at::Tensor ws = workspace(x, wsb);
  SparcMixerBwdArgs a = {};
  a.x = x.data_ptr();
  a.y = yc.data_ptr();
  a.dy = dy.data_ptr();
  a.dx = dx.data_ptr();
  a.nu_log = p[0].data_ptr<float>();
  a.theta_log = p[1].data_ptr<float>();
  a.phase_direction = p[2].data_ptr<float>();
  a.radial_direction = p[3].data_ptr<float>();
  a.write_log_gain = p[4].data_ptr<float>();
  a.write_phase_response = p[5].data_ptr<float>();
  a.write_radial_response = p[6].data_ptr<float>();
  const at::Tensor cc = carry.contiguous(), ct = controls.contiguous();
  a.carry = cc.data_ptr<float>();
  a.controls = ct.data_ptr<float>();
  at::Tensor st;
  if (states.has_value()) {
    TORCH_CHECK(states->sizes() == x.sizes() && states->scalar_type() == x.scalar_type(),
                "mixer_backward: states must be the forward's [batch, length, width] states");
    st = states->contiguous();
    a.states = st.data_ptr();
  }
  a.grad_nu_log = g[0].data_ptr<float>();
  a.grad_theta_log = g[1].data_ptr<float>();
  a.grad_phase_direction = g[2].data_ptr<float>();
  a.grad_radial_direction = g[3].data_ptr<float>();
  a.grad_write_log_gain = g[4].data_ptr<float>();
  a.grad_energy_response = g[5].data_ptr<float>();
  a.grad_write_phase_response = g[6].data_ptr<float>();
  a.grad_write_radial_response = g[7].data_ptr<float>();
  a.workspace = ws.data_ptr();
  a.workspace_bytes = wsb;
  a.batch = B;
  a.length = T;
  a.width = (int)W;
  a.dtype = dt;
  check(sparc_mixer_backward(&a, stream_of(x)), "sparc_mixer_backward");
  std::vector<at::Tensor> out = {dx};
  out.insert(out.end(), g.begin(), g.end());
  return out;
}

// One decode step (forward/decode.py:11-55): (y, new_state_r, new_state_i).
std::tuple<at::Tensor, at::Tensor, at::Tensor> decode_step(
    const at::Tensor& x_in, const at::Tensor& state_r, const at::Tensor& state_i, const at::Tensor& nu_log,
    const at::Tensor& theta_log, const at::Tensor& phase_direction, const at::Tensor& radial_direction,
    const at::Tensor& write_log_gain, const at::Tensor& write_phase_response, const at::Tensor& write_radial_response) {
  TORCH_CHECK(x_in.is_cuda() && x_in.dim() == 2, "decode_step: x must be a CUDA [batch, width] tensor");
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor x = x_in.contiguous();
  const int64_t B = x.size(0), W = x.size(1), M = W / 2;
  const at::Tensor sr = f32(state_r), si = f32(state_i);
  const at::Tensor p[7] = {f32(nu_log), f32(theta_log), f32(phase_direction), f32(radial_direction),
                           f32(write_log_gain), f32(write_phase_response), f32(write_radial_response)};
  at::Tensor y = at::empty_like(x);
  auto fo = x.options().dtype(at::kFloat);
  at::Tensor nr = at::empty({B, M}, fo), ni = at::empty({B, M}, fo);
  SparcDecodeArgs a = {};
  a.x = x.data_ptr();
  a.y = y.data_ptr();
  a.state_r = sr.data_ptr<float>();
  a.state_i = si.data_ptr<float>();
  a.new_state_r = nr.data_ptr<float>();
  a.new_state_i = ni.data_ptr<float>();
  a.nu_log = p[0].data_ptr<float>();
  a.theta_log = p[1].data_ptr<float>();
  a.phase_direction = p[2].data_ptr<float>();
  a.radial_direction = p[3].data_ptr<float>();
  a.write_log_gain = p[4].data_ptr<float>();
  a.write_phase_response = p[5].data_ptr<float>();
  a.write_radial_response = p[6].data_ptr<float>();
  a.batch = B;
  a.width = (int)W;
  a.dtype = dtype_code(x);
  check(sparc_decode_step(&a, stream_of(x)), "sparc_decode_step");
  return {y, nr, ni};
}

// real_scan / real_chunk_scan forward (backward/scan.py:793-884): (out, carry, last). a keeps
// its own dtype (widened to float32 in the kernel); out has b's dtype.
std::tuple<at::Tensor, at::Tensor, at::Tensor> real_scan_forward(const at::Tensor& a_in, const at::Tensor& b_in) {
  TORCH_CHECK(a_in.is_cuda() && a_in.dim() == 3 && b_in.sizes() == a_in.sizes(),
              "real_scan_forward: a and b must be CUDA [batch, length, channels] tensors of one shape");
  c10::cuda::CUDAGuard guard(a_in.device());
  const at::Tensor a = a_in.contiguous(), b = b_in.contiguous();
  const int64_t B = a.size(0), L = a.size(1), D = a.size(2);
  const int dt = dtype_code(b), adt = dtype_code(a);
  auto fo = a.options().dtype(at::kFloat);
  at::Tensor out = at::empty_like(b);
  at::Tensor carry = at::empty({B, sparc_real_carry_chunks(L), D}, fo);
  at::Tensor last = at::empty({B, D}, fo);
  const size_t wsb = sparc_real_workspace_bytes(B, L, D, dt);
  TORCH_CHECK(wsb > 0, "real_scan_forward: unsupported shape (", sparc_last_error(), ")");
  at::Tensor ws = workspace(a, wsb);
  SparcRealFwdArgs r = {};
  r.a = a.data_ptr();
  r.b = b.data_ptr();
  r.out = out.data_ptr();
  r.last = last.data_ptr<float>();
  r.carry = carry.data_ptr<float>();
  r.workspace = ws.data_ptr();
  r.workspace_bytes = wsb;
  r.batch = B;
  r.length = L;
  r.channels = D;
  r.dtype = dt;
  r.a_dtype = adt;
  check(sparc_real_scan_forward(&r, stream_of(a)), "sparc_real_scan_forward");
  return {out, carry, last};
}

// Its backward: (grad_a in a's dtype, grad_b in b's).
std::tuple<at::Tensor, at::Tensor> real_scan_backward(const at::Tensor& a_in, const at::Tensor& b_in,
                                                      const at::Tensor& g_in, const at::Tensor& carry) {
  TORCH_CHECK(a_in.is_cuda() && a_in.dim() == 3 && b_in.sizes() == a_in.sizes() && g_in.sizes() == a_in.sizes(),
              "real_scan_backward: a, b and grad_out must be CUDA [batch, length, channels] tensors of one shape");
  c10::cuda::CUDAGuard guard(a_in.device());
  const at::Tensor a = a_in.contiguous(), b = b_in.contiguous(), g = g_in.to(b.scalar_type()).contiguous(),
                   cc = carry.contiguous();
  const int64_t B = a.size(0), L = a.size(1), D = a.size(2);
  const int dt = dtype_code(b), adt = dtype_code(a);
  at::Tensor ga = at::empty_like(a), gb = at::empty_like(b);
  const size_t wsb = sparc_real_workspace_bytes(B, L, D, dt);
  TORCH_CHECK(wsb > 0, "real_scan_backward: unsupported shape (", sparc_last_error(), ")");
  at::Tensor ws = workspace(a, wsb);
  SparcRealBwdArgs r = {};
  r.a = a.data_ptr();
  r.b = b.data_ptr();
  r.grad_out = g.data_ptr();
  r.carry = cc.data_ptr<float>();
  r.grad_a = ga.data_ptr();
  r.grad_b = gb.data_ptr();
  r.workspace = ws.data_ptr();
  r.workspace_bytes = wsb;
  r.batch = B;
  r.length = L;
  r.channels = D;
  r.dtype = dt;
  r.a_dtype = adt;
  check(sparc_real_scan_backward(&r, stream_of(a)), "sparc_real_scan_backward");
  return {ga, gb};
}

}  // namespace

TORCH_LIBRARY(sparc_b200, m) {
  m.def("mixer_forward(Tensor x, Tensor nu_log, Tensor theta_log, Tensor phase_direction, Tensor radial_direction, "
        "Tensor write_log_gain, Tensor write_phase_response, Tensor write_radial_response) "
        "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("mixer_backward(Tensor x, Tensor y, Tensor dy, Tensor nu_log, Tensor theta_log, Tensor phase_direction, "
        "Tensor radial_direction, Tensor write_log_gain, Tensor write_phase_response, Tensor write_radial_response, "
        "Tensor carry, Tensor controls, Tensor? states=None) -> Tensor[]");
  m.def("decode_step(Tensor x, Tensor state_r, Tensor state_i, Tensor nu_log, Tensor theta_log, "
        "Tensor phase_direction, Tensor radial_direction, Tensor write_log_gain, Tensor write_phase_response, "
        "Tensor write_radial_response) -> (Tensor, Tensor, Tensor)");
  m.def("real_scan_forward(Tensor a, Tensor b) -> (Tensor, Tensor, Tensor)");
  m.def("real_scan_backward(Tensor a, Tensor b, Tensor grad_out, Tensor carry) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(sparc_b200, CUDA, m) {
  m.impl("mixer_forward", &mixer_forward);
  m.impl("mixer_backward", &mixer_backward);
  m.impl("decode_step", &decode_step);
  m.impl("real_scan_forward", &real_scan_forward);
  m.impl("real_scan_backward", &real_scan_backward);
}
