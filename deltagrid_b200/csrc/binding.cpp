// binding.cpp -- the drop-in module `hsru_delta_cuda` as a compiled torch extension.
//
// Same functions, argument names, defaults and return lists as the reference's
// pybind module (src/cpp/binding.cpp:523-561); each function checks and prepares
// its tensors the way the reference binding does, allocates outputs with torch's
// caching allocator, and calls one C-ABI entry point of libdeltagrid_b200.so
// (include/deltagrid_b200.h) on torch's current stream of the input's device.
// There is no CPU path: a non-CUDA tensor raises, as in the reference.
//
// Errors: argument checks raise RuntimeError with the reference's messages
// ("x must be a CUDA tensor", the dtype-dispatch "not implemented for" text); a
// non-zero dg_status raises deltagrid_b200._lib.DeltaGridError (a RuntimeError).
#include <torch/extension.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "deltagrid_b200.h"

namespace py = pybind11;
using at::Tensor;

namespace {

PyObject* g_error = nullptr;   // deltagrid_b200._lib.DeltaGridError, set at import

[[noreturn]] void raise_status(int st, const char* what) {
    std::string msg = std::string(what) + " failed: " + dg_status_string(st);
    if (st == DG_ERR_CUDA) msg += " (cudaError " + std::to_string(dg_last_cuda_error()) + ")";
    msg += " [status " + std::to_string(st) + "]";
    PyErr_SetString(g_error ? g_error : PyExc_RuntimeError, msg.c_str());
    throw py::error_already_set();
}
inline void check(int st, const char* what) {
    if (st != 0) raise_status(st, what);
}

// binding.cpp:18 -- TORCH_CHECK(x.is_cuda(), #x " must be a CUDA tensor")
inline void check_cuda(const Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

// AT_DISPATCH_FLOATING_TYPES_AND2(Half, BFloat16, ...) of the reference bindings
int dtype_code(const Tensor& t, const char* op) {
    switch (t.scalar_type()) {
    case at::kFloat: return DG_DTYPE_F32;
    case at::kDouble: return DG_DTYPE_F64;
    case at::kHalf: return DG_DTYPE_F16;
    case at::kBFloat16: return DG_DTYPE_BF16;
    default: TORCH_CHECK(false, "\"", op, "\" not implemented for '", c10::toString(t.scalar_type()), "'");
    }
    return -1;
}

// data_ptr<scalar_t>() in the reference raises when a tensor's dtype differs
inline void same_dtype(const Tensor& ref, const char* op, const char* name, const Tensor& t) {
    TORCH_CHECK(t.scalar_type() == ref.scalar_type(), op, ": expected ", name, " to have dtype ",
                c10::toString(ref.scalar_type()), ", got ", c10::toString(t.scalar_type()));
}

inline Tensor contig(const Tensor& t) { return t.is_contiguous() ? t : t.contiguous(); }

inline void* stream_of(const Tensor& t) {
    return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// one int32 device status word per device for the kernels' self-checks; kept for
// the life of the process (never freed, so nothing runs after CUDA shuts down)
Tensor& status_word(const at::Device& dev) {
    static auto* words = new std::unordered_map<int, Tensor>();
    auto it = words->find(dev.index());
    if (it == words->end())
        it = words->emplace(dev.index(), at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(dev))).first;
    return it->second;
}

inline void* ptr_or_null(const Tensor& t) { return t.defined() ? t.data_ptr() : nullptr; }

// ---------------------------------------------------------------------------
// dense
// ---------------------------------------------------------------------------

// binding.cpp:36-113.  Returns [out, s_final, err_out, s_final_f]: err_out (fp32
// residuals) is undefined unless save_for_backward; s_final_f is an fp32 copy of the
// final state when saving a non-fp32 run, else s_final itself.
std::vector<Tensor> forward(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& beta,
                            const Tensor& wk, const Tensor& wq, const Tensor& decay,
                            const c10::optional<Tensor>& s_init, bool save_for_backward, int algo) {
    check_cuda(q, "q");
    check_cuda(k, "k");
    check_cuda(v, "v");
    check_cuda(beta, "beta");
    check_cuda(wk, "wk");
    check_cuda(wq, "wq");
    check_cuda(decay, "decay");
    const Tensor v_c = contig(v), beta_c = contig(beta), wk_c = contig(wk), wq_c = contig(wq),
                 decay_c = contig(decay);
    const int code = dtype_code(v_c, "delta_grid_forward_cuda");
    same_dtype(v_c, "forward", "beta", beta_c);
    same_dtype(v_c, "forward", "wk", wk_c);
    same_dtype(v_c, "forward", "wq", wq_c);
    same_dtype(v_c, "forward", "decay", decay_c);
    TORCH_CHECK(v_c.dim() == 4 && wk_c.dim() == 4, "forward: v and wk must be [B,H,T,*]");
    const int64_t B = v_c.size(0), H = v_c.size(1), T = v_c.size(2), Dh = v_c.size(3), S = wk_c.size(3);
    Tensor s_init_c;
    if (s_init.has_value() && s_init->defined()) {
        check_cuda(*s_init, "s_init.value()");
        s_init_c = contig(*s_init);
        same_dtype(v_c, "forward", "s_init", s_init_c);
    }
    const auto opt = v_c.options();
    Tensor out = at::empty({B, H, T, Dh}, opt);
    Tensor s_final = at::empty({B, H, S, Dh}, opt);
    const bool is_fp32 = v_c.scalar_type() == at::kFloat;
    Tensor err_out, s_final_f = s_final;
    if (save_for_backward) {
        err_out = at::empty({B, H, T, Dh}, opt.dtype(at::kFloat));
        if (!is_fp32) s_final_f = at::empty({B, H, S, Dh}, opt.dtype(at::kFloat));
    }
    const c10::cuda::CUDAGuard guard(v_c.device());
    check(dg_dense_forward_ex2(code, (int)B, (int)H, (int)T, (int)S, (int)Dh, v_c.data_ptr(), beta_c.data_ptr(),
                               wk_c.data_ptr(), wq_c.data_ptr(), decay_c.data_ptr(), decay_c.dim() > 1 ? 1 : 0,
                               ptr_or_null(s_init_c), out.data_ptr(), s_final.data_ptr(),
                               err_out.defined() ? err_out.data_ptr<float>() : nullptr,
                               (save_for_backward && !is_fp32) ? s_final_f.data_ptr<float>() : nullptr,
                               status_word(v_c.device()).data_ptr<int32_t>(), algo, stream_of(v_c)),
          "dg_dense_forward_ex2");
    return {out, s_final, err_out, s_final_f};
}

// binding.cpp:130-203.  Returns [out, s_next].  v, wk, wq and beta may be strided
// over (batch, head) as long as their last dimension is contiguous; outputs take
// q's dtype and device, as in the reference.
std::vector<Tensor> step(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& beta, const Tensor& wk,
                         const Tensor& wq, const Tensor& decay, const Tensor& s_prev) {
    check_cuda(q, "q");
    check_cuda(k, "k");
    check_cuda(v, "v");
    check_cuda(beta, "beta");
    check_cuda(wk, "wk");
    check_cuda(wq, "wq");
    check_cuda(decay, "decay");
    check_cuda(s_prev, "s_prev");
    TORCH_CHECK(v.dim() == 3 && wk.dim() == 3 && wq.dim() == 3 && beta.dim() == 2,
                "step: expected v [B,H,Dh], beta [B,H], wk and wq [B,H,slots]");
    const Tensor v_c = v.stride(2) == 1 ? v : v.contiguous();
    const Tensor wk_c = wk.stride(2) == 1 ? wk : wk.contiguous();
    const Tensor wq_c = wq.stride(2) == 1 ? wq : wq.contiguous();
    const bool dynamic = decay.dim() > 1;
    const Tensor decay_c = (!dynamic && decay.stride(0) != 1) ? decay.contiguous() : decay;
    const Tensor s_prev_c = contig(s_prev);
    const int code = dtype_code(v_c, "delta_grid_step_cuda");
    same_dtype(v_c, "step", "beta", beta);
    same_dtype(v_c, "step", "wk", wk_c);
    same_dtype(v_c, "step", "wq", wq_c);
    same_dtype(v_c, "step", "decay", decay_c);
    same_dtype(v_c, "step", "s_prev", s_prev_c);
    same_dtype(v_c, "step", "out", q);
    const int64_t B = v_c.size(0), H = v_c.size(1), Dh = v_c.size(2), S = wk_c.size(2);
    Tensor out = at::empty({B, H, Dh}, q.options());
    Tensor s_next = at::empty({B, H, S, Dh}, q.options());
    const int64_t d_sb = dynamic ? decay_c.stride(0) : 0, d_sh = dynamic ? decay_c.stride(1) : 1;
    const c10::cuda::CUDAGuard guard(v_c.device());
    check(dg_dense_step(code, (int)B, (int)H, (int)S, (int)Dh, v_c.data_ptr(), v_c.stride(0), v_c.stride(1),
                        beta.data_ptr(), beta.stride(0), beta.stride(1), wk_c.data_ptr(), wk_c.stride(0),
                        wk_c.stride(1), wq_c.data_ptr(), wq_c.stride(0), wq_c.stride(1), decay_c.data_ptr(),
                        dynamic ? 1 : 0, d_sb, d_sh, s_prev_c.data_ptr(), out.data_ptr(), s_next.data_ptr(),
                        stream_of(v_c)),
          "dg_dense_step");
    return {out, s_next};
}

// binding.cpp:223-312.  s_final and err_saved are forward(..., save_for_backward=True)'s
// s_final_f and err_out.  Returns [grad_v, grad_beta, grad_wk, grad_wq, grad_decay,
// grad_s_init]; grad_s_init is undefined unless needs_grad_s_init.  A static [H] decay
// gets the sum over the batch.
std::vector<Tensor> backward(const Tensor& grad_out, const c10::optional<Tensor>& grad_s_final, const Tensor& v,
                             const Tensor& beta, const Tensor& wk, const Tensor& wq, const Tensor& decay,
                             const Tensor& s_final, const Tensor& err_saved, bool needs_grad_s_init) {
    check_cuda(grad_out, "grad_out");
    check_cuda(v, "v");
    check_cuda(beta, "beta");
    check_cuda(wk, "wk");
    check_cuda(wq, "wq");
    check_cuda(decay, "decay");
    check_cuda(s_final, "s_final");
    check_cuda(err_saved, "err_saved");
    const Tensor go_c = contig(grad_out), v_c = contig(v), beta_c = contig(beta), wk_c = contig(wk),
                 wq_c = contig(wq), decay_c = contig(decay);
    const Tensor sf_c = s_final.to(at::kFloat).contiguous(), err_c = err_saved.to(at::kFloat).contiguous();
    const int code = dtype_code(v_c, "delta_grid_backward_cuda");
    same_dtype(v_c, "backward", "grad_out", go_c);
    same_dtype(v_c, "backward", "beta", beta_c);
    same_dtype(v_c, "backward", "wk", wk_c);
    same_dtype(v_c, "backward", "wq", wq_c);
    same_dtype(v_c, "backward", "decay", decay_c);
    const int64_t B = v_c.size(0), H = v_c.size(1), T = v_c.size(2), Dh = v_c.size(3), S = wk_c.size(3);
    Tensor gsf;
    if (grad_s_final.has_value() && grad_s_final->defined()) {
        check_cuda(*grad_s_final, "grad_s_final");
        gsf = contig(*grad_s_final);
        same_dtype(v_c, "backward", "grad_s_final", gsf);
    }
    const bool dynamic = decay_c.dim() > 1;
    Tensor grad_v = at::empty_like(v_c), grad_beta = at::empty_like(beta_c), grad_wk = at::empty_like(wk_c),
           grad_wq = at::empty_like(wq_c);
    Tensor grad_decay = dynamic ? at::empty_like(decay_c) : at::zeros_like(decay_c);
    Tensor grad_s_init;
    if (needs_grad_s_init) grad_s_init = at::empty({B, H, S, Dh}, v_c.options());
    const c10::cuda::CUDAGuard guard(v_c.device());
    const size_t nws = dg_dense_backward_workspace_size((int)B, (int)H, (int)S, (int)Dh);
    Tensor ws;
    if (nws) ws = at::empty({(int64_t)(nws / 4)}, v_c.options().dtype(at::kFloat));
    check(dg_dense_backward(code, (int)B, (int)H, (int)T, (int)S, (int)Dh, go_c.data_ptr(), ptr_or_null(gsf),
                            v_c.data_ptr(), beta_c.data_ptr(), wk_c.data_ptr(), wq_c.data_ptr(), decay_c.data_ptr(),
                            dynamic ? 1 : 0, sf_c.data_ptr<float>(), err_c.data_ptr<float>(), grad_v.data_ptr(),
                            grad_beta.data_ptr(), grad_wk.data_ptr(), grad_wq.data_ptr(), grad_decay.data_ptr(),
                            ptr_or_null(grad_s_init), ws.defined() ? ws.data_ptr<float>() : nullptr,
                            stream_of(v_c)),
          "dg_dense_backward");
    return {grad_v, grad_beta, grad_wk, grad_wq, grad_decay, grad_s_init};
}

// ---------------------------------------------------------------------------
// Sparse Delta-PKM
// ---------------------------------------------------------------------------

inline void check_index(const Tensor& idx, const char* op) {
    TORCH_CHECK(idx.scalar_type() == at::kLong, op, ": expected active_idx to have dtype ",
                c10::toString(at::kLong), ", got ", c10::toString(idx.scalar_type()));
}

// binding.cpp:319-370.  State updated in place; returns [out, state].  A [B,H] decay
// is applied per batch row (the PyTorch path's semantics, memory.py:582-591).
std::vector<Tensor> pkm_step(const Tensor& v, const Tensor& beta, const Tensor& wk, const Tensor& wq,
                             const Tensor& active_idx, const Tensor& decay, const Tensor& state_1m) {
    check_cuda(v, "v");
    check_cuda(beta, "beta");
    check_cuda(wk, "wk");
    check_cuda(wq, "wq");
    check_cuda(active_idx, "active_idx");
    check_cuda(decay, "decay");
    check_cuda(state_1m, "state_1m");
    const Tensor v_c = contig(v), beta_c = contig(beta), wk_c = contig(wk), wq_c = contig(wq),
                 idx_c = contig(active_idx), decay_c = contig(decay);
    Tensor state_c = contig(state_1m);
    const int code = dtype_code(v_c, "delta_pkm_step_cuda");
    same_dtype(v_c, "pkm_step", "beta", beta_c);
    same_dtype(v_c, "pkm_step", "wk", wk_c);
    same_dtype(v_c, "pkm_step", "wq", wq_c);
    same_dtype(v_c, "pkm_step", "decay", decay_c);
    same_dtype(v_c, "pkm_step", "state", state_c);
    check_index(idx_c, "pkm_step");
    const int64_t B = v_c.size(0), H = v_c.size(1), Dh = v_c.size(2), A = wk_c.size(2), total = state_c.size(2);
    Tensor out = at::empty({B, H, Dh}, v_c.options());
    const c10::cuda::CUDAGuard guard(v_c.device());
    check(dg_pkm_step(code, (int)B, (int)H, (int)A, total, (int)Dh, v_c.data_ptr(), beta_c.data_ptr(),
                      wk_c.data_ptr(), wq_c.data_ptr(), idx_c.data_ptr<int64_t>(), decay_c.data_ptr(),
                      decay_c.dim() > 1 ? 1 : 0, state_c.data_ptr(), out.data_ptr(),
                      status_word(v_c.device()).data_ptr<int32_t>(), stream_of(v_c)),
          "dg_pkm_step");
    return {out, state_c};
}

// binding.cpp:375-434 with an explicit kernel (dg_pkm_algo; 0 chooses).  State
// updated in place; returns [out, state, saved_s_act], saved_s_act [B,H,T,A,Dh] the
// rows gathered at each step when save_for_backward, else undefined.
std::vector<Tensor> pkm_forward_algo(const Tensor& v, const Tensor& beta, const Tensor& wk, const Tensor& wq,
                                     const Tensor& active_idx, const Tensor& decay, const Tensor& state,
                                     bool save_for_backward, int algo) {
    check_cuda(v, "v");
    check_cuda(beta, "beta");
    check_cuda(wk, "wk");
    check_cuda(wq, "wq");
    check_cuda(active_idx, "active_idx");
    check_cuda(decay, "decay");
    check_cuda(state, "state");
    const Tensor v_c = contig(v), beta_c = contig(beta), wk_c = contig(wk), wq_c = contig(wq),
                 idx_c = contig(active_idx), decay_c = contig(decay);
    Tensor state_c = contig(state);
    const int code = dtype_code(v_c, "delta_pkm_forward_cuda");
    same_dtype(v_c, "pkm_forward", "beta", beta_c);
    same_dtype(v_c, "pkm_forward", "wk", wk_c);
    same_dtype(v_c, "pkm_forward", "wq", wq_c);
    same_dtype(v_c, "pkm_forward", "decay", decay_c);
    same_dtype(v_c, "pkm_forward", "state", state_c);
    check_index(idx_c, "pkm_forward");
    const int64_t B = v_c.size(0), H = v_c.size(1), T = v_c.size(2), Dh = v_c.size(3), A = wk_c.size(3),
                  total = state_c.size(2);
    Tensor out = at::empty({B, H, T, Dh}, v_c.options());
    Tensor saved;
    if (save_for_backward) saved = at::empty({B, H, T, A, Dh}, v_c.options());
    const c10::cuda::CUDAGuard guard(v_c.device());
    // scratch for kernels that need it (per-row hazard codes), from torch's caching allocator
    const size_t nws = dg_pkm_forward_workspace_size(code, (int)B, (int)H, (int)T, (int)A, total, (int)Dh, algo);
    Tensor ws;
    if (nws) ws = at::empty({(int64_t)nws}, v_c.options().dtype(at::kByte));
    check(dg_pkm_forward_ex(code, (int)B, (int)H, (int)T, (int)A, total, (int)Dh, v_c.data_ptr(), beta_c.data_ptr(),
                            wk_c.data_ptr(), wq_c.data_ptr(), idx_c.data_ptr<int64_t>(), decay_c.data_ptr(),
                            decay_c.dim() > 1 ? 1 : 0, state_c.data_ptr(), out.data_ptr(), ptr_or_null(saved),
                            status_word(v_c.device()).data_ptr<int32_t>(), algo, ptr_or_null(ws), nws,
                            stream_of(v_c)),
          "dg_pkm_forward_ex");
    return {out, state_c, saved};
}

std::vector<Tensor> pkm_forward(const Tensor& v, const Tensor& beta, const Tensor& wk, const Tensor& wq,
                                const Tensor& active_idx, const Tensor& decay, const Tensor& state,
                                bool save_for_backward) {
    return pkm_forward_algo(v, beta, wk, wq, active_idx, decay, state, save_for_backward, DG_PKM_AUTO);
}

// binding.cpp:439-518.  saved_s_act: pkm_forward(..., save_for_backward=True)'s rows.
// Returns [grad_v, grad_beta, grad_wk, grad_wq, grad_decay, grad_state]: grad_state is
// the gradient of the initial state (grad_final_state carried back to step 0);
// grad_decay is undefined unless needs_grad_decay ([B,H,T] for a dynamic decay, else
// [H] summed over the batch -- an output the reference allocates but never writes).
std::vector<Tensor> pkm_backward(const Tensor& grad_out, const Tensor& v, const Tensor& beta, const Tensor& wk,
                                 const Tensor& wq, const Tensor& active_idx, const Tensor& decay,
                                 const Tensor& saved_s_act, int64_t total_slots,
                                 const c10::optional<Tensor>& grad_final_state, bool needs_grad_decay) {
    check_cuda(grad_out, "grad_out");
    check_cuda(v, "v");
    check_cuda(beta, "beta");
    check_cuda(wk, "wk");
    check_cuda(wq, "wq");
    check_cuda(active_idx, "active_idx");
    check_cuda(decay, "decay");
    check_cuda(saved_s_act, "saved_s_act");
    const Tensor go_c = contig(grad_out), v_c = contig(v), beta_c = contig(beta), wk_c = contig(wk),
                 wq_c = contig(wq), idx_c = contig(active_idx), decay_c = contig(decay), sv_c = contig(saved_s_act);
    const int code = dtype_code(v_c, "delta_pkm_backward_cuda");
    same_dtype(v_c, "pkm_backward", "grad_out", go_c);
    same_dtype(v_c, "pkm_backward", "beta", beta_c);
    same_dtype(v_c, "pkm_backward", "wk", wk_c);
    same_dtype(v_c, "pkm_backward", "wq", wq_c);
    same_dtype(v_c, "pkm_backward", "decay", decay_c);
    same_dtype(v_c, "pkm_backward", "saved_s_act", sv_c);
    check_index(idx_c, "pkm_backward");
    const int64_t B = v_c.size(0), H = v_c.size(1), T = v_c.size(2), Dh = v_c.size(3), A = wk_c.size(3);
    const bool dynamic = decay_c.dim() > 1;
    const auto opt = v_c.options();
    Tensor grad_state;
    if (grad_final_state.has_value() && grad_final_state->defined()) {
        check_cuda(*grad_final_state, "grad_final_state");
        grad_state = grad_final_state->clone().contiguous();
        same_dtype(v_c, "pkm_backward", "grad_final_state", grad_state);
    } else {
        grad_state = at::zeros({B, H, total_slots, Dh}, opt);
    }
    Tensor grad_v = at::empty({B, H, T, Dh}, opt), grad_beta = at::empty({B, H, T}, opt),
           grad_wk = at::empty({B, H, T, A}, opt), grad_wq = at::empty({B, H, T, A}, opt);
    Tensor grad_decay;
    if (needs_grad_decay) grad_decay = dynamic ? at::empty({B, H, T}, opt) : at::zeros({H}, opt);
    const c10::cuda::CUDAGuard guard(v_c.device());
    check(dg_pkm_backward(code, (int)B, (int)H, (int)T, (int)A, total_slots, (int)Dh, go_c.data_ptr(),
                          v_c.data_ptr(), beta_c.data_ptr(), wk_c.data_ptr(), wq_c.data_ptr(),
                          idx_c.data_ptr<int64_t>(), decay_c.data_ptr(), dynamic ? 1 : 0, sv_c.data_ptr(),
                          grad_state.data_ptr(), grad_v.data_ptr(), grad_beta.data_ptr(), grad_wk.data_ptr(),
                          grad_wq.data_ptr(), ptr_or_null(grad_decay), status_word(v_c.device()).data_ptr<int32_t>(),
                          stream_of(v_c)),
          "dg_pkm_backward");
    return {grad_v, grad_beta, grad_wk, grad_wq, grad_decay, grad_state};
}

// the device status word the PKM entry points OR their self-check bits into
Tensor device_status_word(int64_t device_index) {
    return status_word(at::Device(at::kCUDA, (c10::DeviceIndex)device_index));
}

}  // namespace

PYBIND11_MODULE(_hsru, m) {
    m.doc() = "DeltaGrid recurrence on B200 (sm_100a): drop-in for the reference extension hsru_delta_cuda";
    g_error = py::object(py::module_::import("deltagrid_b200._lib").attr("DeltaGridError")).release().ptr();

    m.def("forward", &forward, "Dense sequence forward", py::arg("q"), py::arg("k"), py::arg("v"),
          py::arg("beta"), py::arg("wk"), py::arg("wq"), py::arg("decay"), py::arg("s_init") = py::none(),
          py::arg("save_for_backward") = false, py::arg("algo") = (int)DG_DENSE_AUTO);
    m.def("step", &step, "Dense single decode step", py::arg("q"), py::arg("k"), py::arg("v"), py::arg("beta"),
          py::arg("wk"), py::arg("wq"), py::arg("decay"), py::arg("s_prev"));
    m.def("pkm_step", &pkm_step, "Sparse Delta-PKM decode step (state in place)", py::arg("v"), py::arg("beta"),
          py::arg("wk"), py::arg("wq"), py::arg("active_idx"), py::arg("decay"), py::arg("state_1m"));
    m.def("pkm_forward", &pkm_forward, "Sparse Delta-PKM sequence forward (state in place)", py::arg("v"),
          py::arg("beta"), py::arg("wk"), py::arg("wq"), py::arg("active_idx"), py::arg("decay"), py::arg("state"),
          py::arg("save_for_backward") = false);
    m.def("pkm_forward_algo", &pkm_forward_algo, "pkm_forward with an explicit kernel (dg_pkm_algo)", py::arg("v"),
          py::arg("beta"), py::arg("wk"), py::arg("wq"), py::arg("active_idx"), py::arg("decay"), py::arg("state"),
          py::arg("save_for_backward") = false, py::arg("algo") = (int)DG_PKM_AUTO);
    m.def("pkm_backward", &pkm_backward, "Sparse Delta-PKM analytic backward", py::arg("grad_out"), py::arg("v"),
          py::arg("beta"), py::arg("wk"), py::arg("wq"), py::arg("active_idx"), py::arg("decay"),
          py::arg("saved_s_act"), py::arg("total_slots"), py::arg("grad_final_state") = py::none(),
          py::arg("needs_grad_decay") = false);
    m.def("backward", &backward, "Dense analytic backward", py::arg("grad_out"), py::arg("grad_s_final"),
          py::arg("v"), py::arg("beta"), py::arg("wk"), py::arg("wq"), py::arg("decay"), py::arg("s_final"),
          py::arg("err_saved"), py::arg("needs_grad_s_init") = false);
    m.def("device_status_word", &device_status_word, "The int32 device status word of a CUDA device",
          py::arg("device_index"));
}
