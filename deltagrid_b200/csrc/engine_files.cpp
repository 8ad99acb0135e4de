// engine_files.cpp -- the reference C++ engine's two file formats, read and
// written on the host so that its weights and recurrent state can drive the
// GPU recurrence:
//
//   DLG1  weights (DeltaGridBinHeader and the array order of
//         src/cpp/engine/include/deltagrid_internal.h:1-85).  dg_dlg1_layout walks
//         the file in the order the engine's loaders read it -- the float/int8
//         loader dg_load_context_from_file (src/cpp/engine/src/deltagrid_math.cpp:
//         558-761) and the Q16.16 loader deltagrid_init_context_fxp
//         (src/cpp/engine/src/deltagrid_fxp.cpp:503-660) -- and reports every
//         array's byte offset, element count and encoding, so a caller can map
//         the arrays it needs (the memory tier's router and slot projections,
//         decay, q_scale, ...) without copying the rest.
//   DLGS  recurrent state snapshots (dg_save_runtime_state / dg_load_runtime_state,
//         deltagrid_math.cpp:779-844; the Q16.16 twins deltagrid_save_state_fxp /
//         deltagrid_load_state_fxp, deltagrid_fxp.cpp:728-795): a 7 x int32 header
//         (magic, layers, d_model, heads, slots, kernel size, step count), then per
//         layer the conv window [d_model * max(K-1, 1)] and the memory state
//         [heads, slots, d_model / heads], 4-byte elements (fp32 or Q16.16).
//
// Host code only; no CUDA.  Every entry point returns DG_OK or a negative
// dg_status; DG_ERR_FORMAT covers unreadable, truncated or inconsistent files.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "deltagrid_b200.h"

namespace {

constexpr int32_t kDlg1Magic = 0x31474C44;   // 'DLG1'
constexpr int32_t kDlgsMagic = 0x53474C44;   // 'DLGS'
constexpr int32_t kPrecF32 = 0, kPrecInt8 = 1, kPrecFxp = 2;
constexpr int32_t kModelContinuous = 0, kModelLm = 1;
constexpr int32_t kFlagDynamicDecay = 1, kFlagSlotProj = 2, kFlagTiedHead = 4;

struct File {
    FILE* f = nullptr;
    explicit File(const char* path, const char* mode) : f(std::fopen(path, mode)) {}
    ~File() {
        if (f) std::fclose(f);
    }
    bool ok() const { return f != nullptr; }
};

int64_t file_size(FILE* f) {
    if (std::fseek(f, 0, SEEK_END) != 0) return -1;
    const long n = std::ftell(f);
    if (n < 0 || std::fseek(f, 0, SEEK_SET) != 0) return -1;
    return n;
}

// Walks a DLG1 file in load order, recording arrays; the only values it reads
// from the body are the per-block has_memory words and int8 scales.
class Walker {
  public:
    Walker(FILE* f, int64_t size, int32_t pmode, dg_dlg1_array* out, int cap)
        : f_(f), size_(size), pmode_(pmode), out_(out), cap_(cap) {}

    bool failed() const { return failed_; }
    int count() const { return n_; }
    int64_t pos() const { return pos_; }
    void skip(int64_t bytes) { advance(bytes); }

    int32_t read_i32() {
        int32_t v = 0;
        if (pos_ + 4 > size_ || std::fseek(f_, (long)pos_, SEEK_SET) != 0 || std::fread(&v, 4, 1, f_) != 1) {
            failed_ = true;
            return 0;
        }
        pos_ += 4;
        return v;
    }
    // a vector (load_f32_array / load_i32_array): fp32, or Q16.16 in fixed-point files
    void vec(const char* name, int64_t n, int layer = -1, int axis = -1) {
        if (n == 0) return;
        record(name, n, layer, axis, pmode_ == kPrecFxp ? DG_ENC_Q16 : DG_ENC_F32, 1.f, pos_);
        advance(4 * n);
    }
    // one float (or Q16.16) read straight into a struct field: clock_scale, scale_mem, scale_logic
    void scalar(const char* name, int layer) { vec(name, 1, layer); }
    // a weight matrix (load_weight_array): fp32, int8 after an fp32 scale, or Q16.16
    void weight(const char* name, int64_t n, int layer = -1) {
        if (n == 0) return;
        if (pmode_ == kPrecInt8) {
            float scale = 1.f;
            if (pos_ + 4 > size_ || std::fseek(f_, (long)pos_, SEEK_SET) != 0 || std::fread(&scale, 4, 1, f_) != 1) {
                failed_ = true;
                return;
            }
            pos_ += 4;
            record(name, n, layer, -1, DG_ENC_Q8, scale, pos_);
            advance(n);
        } else {
            vec(name, n, layer);
        }
    }

  private:
    void advance(int64_t bytes) {
        if (bytes < 0 || pos_ + bytes > size_) failed_ = true;
        else pos_ += bytes;
    }
    void record(const char* name, int64_t n, int layer, int axis, int enc, float scale, int64_t off) {
        if (out_ && n_ < cap_) {
            dg_dlg1_array& a = out_[n_];
            std::memset(&a, 0, sizeof(a));
            std::strncpy(a.name, name, sizeof(a.name) - 1);
            a.layer = layer;
            a.axis = axis;
            a.encoding = enc;
            a.scale = scale;
            a.offset = off;
            a.count = n;
        }
        ++n_;
    }

    FILE* f_;
    int64_t size_;
    int32_t pmode_;
    dg_dlg1_array* out_;
    int cap_;
    int n_ = 0;
    int64_t pos_ = 0;
    bool failed_ = false;
};

bool dims_ok(int64_t a, int64_t b, int64_t c = 1) { return a >= 0 && b >= 0 && c >= 0 && a * b * c < (int64_t(1) << 40); }

}  // namespace

extern "C" {

int dg_dlg1_layout(const char* path, dg_dlg1_header* hdr, int32_t* grid_dim, int max_axes, dg_dlg1_array* arrays,
                   int max_arrays, int* n_arrays) {
    if (!path || !hdr || !n_arrays || max_axes < 0 || max_arrays < 0) return DG_ERR_INVALID_ARGUMENT;
    File file(path, "rb");
    if (!file.ok()) return DG_ERR_FORMAT;
    const int64_t size = file_size(file.f);
    if (size < (int64_t)sizeof(dg_dlg1_header)) return DG_ERR_FORMAT;
    dg_dlg1_header h;
    if (std::fread(&h, sizeof(h), 1, file.f) != 1) return DG_ERR_FORMAT;
    if (h.magic != kDlg1Magic) return DG_ERR_FORMAT;
    if (h.precision_mode != kPrecF32 && h.precision_mode != kPrecInt8 && h.precision_mode != kPrecFxp)
        return DG_ERR_FORMAT;
    if (h.model_type != kModelContinuous && h.model_type != kModelLm) return DG_ERR_FORMAT;
    if (h.num_layers < 0 || h.d_model <= 0 || h.num_heads <= 0 || h.d_model % h.num_heads != 0 ||
        h.kernel_size < 0 || h.num_axes < 0 || h.num_axes > DG_DLG1_MAX_AXES || h.actual_slots < 0 ||
        h.input_or_vocab < 0 || h.output_dim < 0 || h.forecast_horizon < 0)
        return DG_ERR_FORMAT;
    *hdr = h;
    const int64_t L = h.num_layers, D = h.d_model, H = h.num_heads, Dh = D / H, K = h.kernel_size;
    const bool dyn = (h.flags & kFlagDynamicDecay) != 0, slot_proj = (h.flags & kFlagSlotProj) != 0;
    const bool lm = h.model_type == kModelLm;
    if (!dims_ok(3 * D + H, D) || !dims_ok(h.input_or_vocab, D) || !dims_ok(h.output_dim, D, h.forecast_horizon + 1) ||
        !dims_ok(h.actual_slots, Dh))
        return DG_ERR_FORMAT;

    Walker w(file.f, size, h.precision_mode, arrays, max_arrays);
    w.skip(sizeof(dg_dlg1_header));
    std::vector<int32_t> grid;
    for (int a = 0; a < h.num_axes; ++a) {
        const int32_t g = w.read_i32();
        if (g <= 0 || !dims_ok(g, Dh)) return DG_ERR_FORMAT;
        grid.push_back(g);
        if (grid_dim && a < max_axes) grid_dim[a] = g;
    }
    if (w.failed()) return DG_ERR_FORMAT;

    // 1. input encoder (deltagrid_math.cpp:617-623; deltagrid_fxp.cpp:547-548)
    if (lm) {
        w.weight("input_weight", (int64_t)h.input_or_vocab * D);
    } else {
        w.weight("input_weight", D * (int64_t)h.input_or_vocab);
        w.vec("input_bias", D);
    }
    // 2. blocks (deltagrid_math.cpp:629-690; deltagrid_fxp.cpp:553-608)
    for (int l = 0; l < (int)L && !w.failed(); ++l) {
        const int32_t has_mem = w.read_i32();
        w.vec("div_term", D / 2, l);
        w.scalar("clock_scale", l);
        w.vec("conv1d_weight", D * K, l);
        w.vec("conv1d_bias", D, l);
        w.vec("norm_conv.weight", D, l);
        w.vec("norm_conv.bias", D, l);
        if (has_mem) {
            w.scalar("memory.scale_mem", l);
            w.weight("memory.proj_qkv_beta", (3 * D + H) * D, l);
            w.vec("memory.q_scale", H, l);
            w.vec("memory.beta_bias", H, l);
            w.vec("memory.decay", H, l);
            if (dyn) {
                w.weight("memory.proj_alpha_weight", H * D, l);
                w.vec("memory.proj_alpha_bias", H, l);
            }
            if (h.num_axes > 0) {
                for (int a = 0; a < h.num_axes; ++a) {
                    w.vec("memory.axes_proj_k", grid[a] * Dh, l, a);
                    w.vec("memory.axes_proj_q", grid[a] * Dh, l, a);
                }
            } else if (slot_proj) {
                w.vec("memory.slot_proj_k", (int64_t)h.actual_slots * Dh, l);
                w.vec("memory.slot_proj_q", (int64_t)h.actual_slots * Dh, l);
            }
            w.weight("memory.out_proj", D * D, l);
            w.vec("memory.norm.weight", D, l);
            w.vec("memory.norm.bias", D, l);
        }
        w.scalar("scale_logic", l);
        w.weight("ffn_fc1_weight", 2 * D * D, l);
        w.vec("ffn_fc1_bias", 2 * D, l);
        w.weight("ffn_fc2_weight", D * D, l);
        w.vec("ffn_fc2_bias", D, l);
        w.vec("norm_ffn.weight", D, l);
        w.vec("norm_ffn.bias", D, l);
    }
    // 3. readout (deltagrid_math.cpp:693-721; deltagrid_fxp.cpp:610-620)
    w.vec("final_norm.weight", D);
    w.vec("final_norm.bias", D);
    if (lm) {
        // the exporter writes no head when it is tied (export_deltagrid_binary.py:220-222)
        if (!(h.flags & kFlagTiedHead)) w.weight("head_weight", (int64_t)h.output_dim * D);
    } else {
        w.weight("head_weight", (int64_t)h.output_dim * D);
        w.vec("head_bias", h.output_dim);
        if (h.forecast_horizon > 0) {
            w.weight("forecast_fc1_weight", D * D);
            w.vec("forecast_fc1_bias", D);
            w.weight("forecast_fc2_weight", (int64_t)h.forecast_horizon * h.output_dim * D);
            w.vec("forecast_fc2_bias", (int64_t)h.forecast_horizon * h.output_dim);
        }
    }
    if (w.failed() || w.pos() != size) return DG_ERR_FORMAT;    // truncated, or bytes the loaders never read
    *n_arrays = w.count();
    return (arrays && w.count() > max_arrays) ? DG_ERR_WORKSPACE : DG_OK;
}

int dg_dlgs_read_header(const char* path, dg_dlgs_header* h) {
    if (!path || !h) return DG_ERR_INVALID_ARGUMENT;
    File file(path, "rb");
    if (!file.ok()) return DG_ERR_FORMAT;
    const int64_t size = file_size(file.f);
    int32_t w[7];
    if (size < 28 || std::fread(w, 4, 7, file.f) != 7 || w[0] != kDlgsMagic) return DG_ERR_FORMAT;
    dg_dlgs_header r{w[1], w[2], w[3], w[4], w[5], w[6]};
    if (r.num_layers < 0 || r.d_model <= 0 || r.num_heads <= 0 || r.d_model % r.num_heads != 0 ||
        r.actual_slots < 0 || r.kernel_size < 0)
        return DG_ERR_FORMAT;
    if (size != 28 + (int64_t)r.num_layers * 4 * (int64_t)(dg_dlgs_conv_elems(&r) + dg_dlgs_mem_elems(&r)))
        return DG_ERR_FORMAT;
    *h = r;
    return DG_OK;
}

size_t dg_dlgs_conv_elems(const dg_dlgs_header* h) {
    const int64_t hist = h->kernel_size > 1 ? h->kernel_size - 1 : 1;     // deltagrid_math.cpp:799
    return (size_t)((int64_t)h->d_model * hist);
}

size_t dg_dlgs_mem_elems(const dg_dlgs_header* h) {
    return (size_t)((int64_t)h->num_heads * h->actual_slots * (h->d_model / h->num_heads));
}

int dg_dlgs_read_layer(const char* path, const dg_dlgs_header* expect, int layer, void* conv_state, void* mem_state) {
    if (!path || !expect || layer < 0 || layer >= expect->num_layers) return DG_ERR_INVALID_ARGUMENT;
    dg_dlgs_header h;
    const int rc = dg_dlgs_read_header(path, &h);
    if (rc != DG_OK) return rc;
    // the engine refuses a snapshot of another shape (deltagrid_math.cpp:827-831); the step count may differ
    if (h.num_layers != expect->num_layers || h.d_model != expect->d_model || h.num_heads != expect->num_heads ||
        h.actual_slots != expect->actual_slots || h.kernel_size != expect->kernel_size)
        return DG_ERR_FORMAT;
    const int64_t nc = (int64_t)dg_dlgs_conv_elems(&h), nm = (int64_t)dg_dlgs_mem_elems(&h);
    File file(path, "rb");
    if (!file.ok()) return DG_ERR_FORMAT;
    const int64_t off = 28 + (int64_t)layer * 4 * (nc + nm);
    if (std::fseek(file.f, (long)off, SEEK_SET) != 0) return DG_ERR_FORMAT;
    if (conv_state) {
        if (std::fread(conv_state, 4, (size_t)nc, file.f) != (size_t)nc) return DG_ERR_FORMAT;
    } else if (std::fseek(file.f, (long)(4 * nc), SEEK_CUR) != 0) {
        return DG_ERR_FORMAT;
    }
    if (mem_state && std::fread(mem_state, 4, (size_t)nm, file.f) != (size_t)nm) return DG_ERR_FORMAT;
    return DG_OK;
}

int dg_dlgs_write(const char* path, const dg_dlgs_header* h, const void* const* conv_layers,
                  const void* const* mem_layers) {
    if (!path || !h || h->num_layers < 0 || h->d_model <= 0 || h->num_heads <= 0 || h->d_model % h->num_heads != 0 ||
        h->actual_slots < 0 || h->kernel_size < 0)
        return DG_ERR_INVALID_ARGUMENT;
    if (h->num_layers > 0 && (!conv_layers || !mem_layers)) return DG_ERR_INVALID_ARGUMENT;
    for (int l = 0; l < h->num_layers; ++l)
        if (!conv_layers[l] || !mem_layers[l]) return DG_ERR_INVALID_ARGUMENT;
    File file(path, "wb");
    if (!file.ok()) return DG_ERR_FORMAT;
    const int32_t w[7] = {kDlgsMagic, h->num_layers, h->d_model, h->num_heads, h->actual_slots, h->kernel_size,
                          h->step_count};
    if (std::fwrite(w, 4, 7, file.f) != 7) return DG_ERR_FORMAT;
    const size_t nc = dg_dlgs_conv_elems(h), nm = dg_dlgs_mem_elems(h);
    for (int l = 0; l < h->num_layers; ++l) {
        if (std::fwrite(conv_layers[l], 4, nc, file.f) != nc) return DG_ERR_FORMAT;
        if (std::fwrite(mem_layers[l], 4, nm, file.f) != nm) return DG_ERR_FORMAT;
    }
    return std::fflush(file.f) == 0 ? DG_OK : DG_ERR_FORMAT;
}

}  // extern "C"
