// Torch-facing fast path of the CUDA engines: the four whole-slice entry
// points of the C ABI (cqt_analysis, cqt_synthesis, cqt_adj_analysis,
// cqt_adj_synthesis) called from C++ with torch's current stream, and
// TrainableCQT's fwd / bwd as C++ autograd functions whose backward nodes run
// the transposes without entering Python.  The C-ABI library stays the only
// place with device code; this module receives its function pointers from the
// Python loader (no link-time dependency) and only moves tensors in and out.
//
// Mirrors trainable.py:141-191 of the reference (TrainableCQT.fwd / bwd: the
// forward returns per-group complex views, the backward of the analysis is
// the transpose of the analysis, that of the synthesis the transpose of the
// synthesis, nothing saved for backward).
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

constexpr int64_t kDefaultN = 65536;
constexpr int kLayoutPlanar = 0;    // CQT_LAYOUT_PLANAR
constexpr int kLayoutComplex = 1;   // CQT_LAYOUT_COMPLEX
constexpr int64_t kWsHeader = 256;  // workspace header (the wait-status word)

// cqt_analysis / cqt_adj_synthesis: signal first
using FnSignalFirst = int (*)(const void*, const float*, float*, float*, int, int, void*,
                              size_t, void*);
// cqt_synthesis / cqt_adj_analysis: coefficients first
using FnCoefFirst = int (*)(const void*, const float*, const float*, int, float*, int, void*,
                            size_t, void*);
using FnWorkspace = size_t (*)(const void*, int);
// cqt_synthesis_sqerr / cqt_adj_synthesis_sqerr (the fused MSE loss)
using FnSynSqErr = int (*)(const void*, const float*, const float*, int, float*, const float*,
                           float*, float, int, void*, size_t, void*);
using FnAdjSynSqErr = int (*)(const void*, const float*, const float*, float, const float*,
                              float*, float*, int, int, void*, size_t, void*);
using FnLastError = const char* (*)();

// One filterbank's device tables on one device, with a grow-only workspace.
// Held by intrusive pointer from Python and from every autograd node that
// may still call it; it keeps the Python owner of the tables alive.
struct Ops : torch::CustomClassHolder {
    const void* tables = nullptr;
    c10::DeviceIndex device = 0;
    int64_t ncoef = 0;
    int64_t kN = kDefaultN;   // samples per slice (65536 or 32768)
    FnSignalFirst an = nullptr, adj_syn = nullptr;
    FnCoefFirst syn = nullptr, adj_an = nullptr;
    FnWorkspace ws_bytes = nullptr;
    FnLastError last_error = nullptr;
    FnSynSqErr syn_sqerr = nullptr;
    FnAdjSynSqErr adj_syn_sqerr = nullptr;
    PyObject* owner = nullptr;         // Python object owning `tables` (strong ref)
    at::Tensor ws;
    std::vector<at::Tensor> retired;   // outgrown workspaces: captured graphs may address them
    std::unordered_map<int64_t, size_t> need;
    std::vector<int64_t> sizes, bins, lens;   // per group: b * M, b, M
    int64_t ngroups = 0;                       // octave groups (the rest are side groups)
    // the heap and views of the last fwd, held weakly, so that bwd can
    // recognise untouched views by identity
    c10::weak_intrusive_ptr<c10::TensorImpl, c10::UndefinedTensorImpl> last_h{
        c10::intrusive_ptr<c10::TensorImpl, c10::UndefinedTensorImpl>()};
    std::vector<c10::weak_intrusive_ptr<c10::TensorImpl, c10::UndefinedTensorImpl>> last_v;

    ~Ops() override {
        if (owner && Py_IsInitialized()) {
            pybind11::gil_scoped_acquire gil;
            Py_DECREF(owner);
        }
    }

    void check(int rc, const char* what) const {
        if (rc != 0)
            TORCH_CHECK(false, what, " failed (", rc, "): ", last_error ? last_error() : "");
    }

    void* workspace(int64_t batch, size_t* bytes) {
        auto it = need.find(batch);
        size_t n;
        if (it == need.end()) {
            n = ws_bytes(tables, (int)batch);
            need.emplace(batch, n);
        } else {
            n = it->second;
        }
        if (!ws.defined() || (size_t)ws.numel() < n) {
            if (ws.defined()) retired.push_back(ws);
            ws = at::empty({(int64_t)std::max<size_t>(n, kWsHeader)},
                           at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device));
            ws.narrow(0, 0, kWsHeader).zero_();   // the wait-status header
        }
        *bytes = (size_t)ws.numel();
        return ws.data_ptr();
    }

    void* stream() const { return at::cuda::getCurrentCUDAStream(device).stream(); }

    at::Tensor signal(const at::Tensor& t, const char* name) const {
        TORCH_CHECK_VALUE(t.defined() && t.is_cuda() && t.get_device() == device, name,
                          " must be a tensor on cuda:", (int)device);
        TORCH_CHECK_TYPE(t.scalar_type() == at::kFloat, name, " must be float32, got ",
                         t.scalar_type());
        TORCH_CHECK_VALUE(t.dim() == 2 && t.size(1) == kN, name, " must be [B, ", kN,
                          "], got ", t.sizes());
        at::Tensor c = t.contiguous();
        // the engines move signals as float2 / float4 vectors
        return (reinterpret_cast<uintptr_t>(c.data_ptr()) & 15u) ? c.clone() : c;
    }

    at::Tensor coef(const at::Tensor& t, const char* name) const {
        TORCH_CHECK_VALUE(t.defined() && t.is_cuda() && t.get_device() == device, name,
                          " must be a tensor on cuda:", (int)device);
        TORCH_CHECK_TYPE(t.scalar_type() == at::kComplexFloat, name,
                         " must be complex64, got ", t.scalar_type());
        TORCH_CHECK_VALUE(t.dim() == 2 && t.size(1) == ncoef, name, " must be [B, ", ncoef,
                          "], got ", t.sizes());
        return t.resolve_conj().contiguous();
    }

    // a float32 [B, ncoef] coefficient plane on this device; `out` planes
    // are written in place, so they must already be contiguous
    at::Tensor plane(const at::Tensor& t, const char* name, int64_t B, bool out) const {
        TORCH_CHECK_VALUE(t.defined() && t.is_cuda() && t.get_device() == device,
                          "coefficient plane ", name, " must be float32 on cuda:", (int)device);
        TORCH_CHECK_VALUE(t.scalar_type() == at::kFloat, "coefficient plane ", name,
                          " must be float32 on cuda:", (int)device);
        TORCH_CHECK_VALUE(t.dim() == 2 && t.size(1) == ncoef && (B < 0 || t.size(0) == B),
                          "coefficient plane ", name, " must be [B, ", ncoef, "]");
        if (out) {
            TORCH_CHECK_VALUE(t.is_contiguous(), "coefficient plane ", name,
                              " must be contiguous");
            return t;
        }
        return t.contiguous();
    }

    struct DeviceSwitch {   // switches only when the current device differs
        c10::optional<c10::cuda::CUDAGuard> g;
        explicit DeviceSwitch(c10::DeviceIndex d) {
            if (c10::cuda::current_device() != d) g.emplace(d);
        }
    };

    at::Tensor analysis(const at::Tensor& x_) {
        at::Tensor x = signal(x_, "x");
        DeviceSwitch sw(device);
        const int64_t B = x.size(0);
        at::Tensor out = at::empty({B, ncoef}, x.options().dtype(at::kComplexFloat));
        size_t wb;
        void* w = workspace(B, &wb);
        check(an(tables, x.data_ptr<float>(), reinterpret_cast<float*>(out.data_ptr()), nullptr,
                 kLayoutComplex, (int)B, w, wb, stream()),
              "cqt_analysis");
        return out;
    }

    // planar layout (FusedOctCQT): results go into the caller's tensors
    void analysis_planar(const at::Tensor& x_, const at::Tensor& kr_, const at::Tensor& ki_) {
        at::Tensor x = signal(x_, "x");
        const int64_t B = x.size(0);
        at::Tensor kr = plane(kr_, "re", B, true), ki = plane(ki_, "im", B, true);
        DeviceSwitch sw(device);
        size_t wb;
        void* w = workspace(B, &wb);
        check(an(tables, x.data_ptr<float>(), kr.data_ptr<float>(), ki.data_ptr<float>(),
                 kLayoutPlanar, (int)B, w, wb, stream()),
              "cqt_analysis");
    }

    void synthesis_planar(const at::Tensor& kr_, const at::Tensor& ki_, const at::Tensor& y) {
        at::Tensor kr = plane(kr_, "re", -1, false);
        const int64_t B = kr.size(0);
        at::Tensor ki = plane(ki_, "im", B, false);
        TORCH_CHECK_VALUE(y.defined() && y.is_cuda() && y.get_device() == device &&
                              y.scalar_type() == at::kFloat && y.dim() == 2 &&
                              y.size(0) == B && y.size(1) == kN && y.is_contiguous(),
                          "y must be a contiguous float32 [B, ", kN, "] tensor on cuda:",
                          (int)device);
        DeviceSwitch sw(device);
        size_t wb;
        void* w = workspace(B, &wb);
        check(syn(tables, kr.data_ptr<float>(), ki.data_ptr<float>(), kLayoutPlanar,
                  y.data_ptr<float>(), (int)B, w, wb, stream()),
              "cqt_synthesis");
    }

    at::Tensor synthesis(const at::Tensor& c_) {
        at::Tensor c = coef(c_, "coefficients");
        DeviceSwitch sw(device);
        const int64_t B = c.size(0);
        at::Tensor out = at::empty({B, kN}, c.options().dtype(at::kFloat));
        size_t wb;
        void* w = workspace(B, &wb);
        check(syn(tables, reinterpret_cast<const float*>(c.data_ptr()), nullptr, kLayoutComplex,
                  out.data_ptr<float>(), (int)B, w, wb, stream()),
              "cqt_synthesis");
        return out;
    }

    at::Tensor adj_analysis(const at::Tensor& g_) {
        at::Tensor g = coef(g_, "coefficient gradient");
        DeviceSwitch sw(device);
        const int64_t B = g.size(0);
        at::Tensor out = at::empty({B, kN}, g.options().dtype(at::kFloat));
        size_t wb;
        void* w = workspace(B, &wb);
        check(adj_an(tables, reinterpret_cast<const float*>(g.data_ptr()), nullptr,
                     kLayoutComplex, out.data_ptr<float>(), (int)B, w, wb, stream()),
              "cqt_adj_analysis");
        return out;
    }

    // synthesis + the squared-error sum against `target`: (loss = mean of
    // (y - target)^2 as a 0-dim float32 tensor, y)
    std::vector<at::Tensor> synthesis_sqerr(const at::Tensor& c_, const at::Tensor& target_) {
        at::Tensor c = coef(c_, "coefficients");
        const int64_t B = c.size(0);
        at::Tensor tgt = signal(target_, "target");
        TORCH_CHECK_VALUE(tgt.size(0) == B, "target must be [", B, ", ", kN, "], got ",
                          tgt.sizes());
        DeviceSwitch sw(device);
        at::Tensor y = at::empty({B, kN}, c.options().dtype(at::kFloat));
        at::Tensor loss = at::empty({}, c.options().dtype(at::kFloat));
        size_t wb;
        void* w = workspace(B, &wb);
        const float scale = B > 0 ? (float)(1.0 / ((double)B * (double)kN)) : 0.f;
        check(syn_sqerr(tables, reinterpret_cast<const float*>(c.data_ptr()), nullptr,
                        kLayoutComplex, y.data_ptr<float>(), tgt.data_ptr<float>(),
                        loss.data_ptr<float>(), scale, (int)B, w, wb, stream()),
              "cqt_synthesis_sqerr");
        return {loss, y, tgt};
    }

    // transpose of the synthesis applied to scale * (*g) * (y - target)
    at::Tensor adj_synthesis_sqerr(const at::Tensor& y, const at::Tensor& tgt, float scale,
                                   const at::Tensor& g) {
        DeviceSwitch sw(device);
        const int64_t B = y.size(0);
        at::Tensor out = at::empty({B, ncoef}, y.options().dtype(at::kComplexFloat));
        size_t wb;
        void* w = workspace(B, &wb);
        check(adj_syn_sqerr(tables, y.data_ptr<float>(), tgt.data_ptr<float>(), scale,
                            g.data_ptr<float>(), reinterpret_cast<float*>(out.data_ptr()),
                            nullptr, kLayoutComplex, (int)B, w, wb, stream()),
              "cqt_adj_synthesis_sqerr");
        return out;
    }

    at::Tensor adj_synthesis(const at::Tensor& gy_) {
        at::Tensor gy = signal(gy_, "signal gradient");
        DeviceSwitch sw(device);
        const int64_t B = gy.size(0);
        at::Tensor out = at::empty({B, ncoef}, gy.options().dtype(at::kComplexFloat));
        size_t wb;
        void* w = workspace(B, &wb);
        check(adj_syn(tables, gy.data_ptr<float>(), reinterpret_cast<float*>(out.data_ptr()),
                      nullptr, kLayoutComplex, (int)B, w, wb, stream()),
              "cqt_adj_synthesis");
        return out;
    }
};

Ops* ops_of(const torch::autograd::AutogradContext* ctx) {
    return static_cast<Ops*>(ctx->saved_data.at("ops").toCapsule().get());
}

// analysis with the transpose of the analysis as its backward
struct AnalysisFn : public torch::autograd::Function<AnalysisFn> {
    static at::Tensor forward(torch::autograd::AutogradContext* ctx, const at::Tensor& x,
                              const c10::intrusive_ptr<Ops>& ops) {
        ctx->saved_data["ops"] = c10::IValue::make_capsule(ops);
        return ops->analysis(x);
    }
    static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                   torch::autograd::variable_list g) {
        if (!g[0].defined()) return {at::Tensor(), at::Tensor()};
        return {ops_of(ctx)->adj_analysis(g[0]), at::Tensor()};
    }
};

// synthesis with the transpose of the synthesis as its backward
struct SynthesisFn : public torch::autograd::Function<SynthesisFn> {
    static at::Tensor forward(torch::autograd::AutogradContext* ctx, const at::Tensor& c,
                              const c10::intrusive_ptr<Ops>& ops) {
        ctx->saved_data["ops"] = c10::IValue::make_capsule(ops);
        return ops->synthesis(c);
    }
    static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                   torch::autograd::variable_list g) {
        if (!g[0].defined()) return {at::Tensor(), at::Tensor()};
        return {ops_of(ctx)->adj_synthesis(g[0]), at::Tensor()};
    }
};

// synthesis + mean squared error against a target: outputs (loss, y), y not
// differentiable (it is a by-product for the caller); the backward runs the
// transpose of the synthesis with dL/dy = 2 dL/dloss (y - target) / n formed
// inside the kernel's load -- no elementwise loss kernels between the engines
struct SynthesisMSEFn : public torch::autograd::Function<SynthesisMSEFn> {
    static torch::autograd::variable_list forward(torch::autograd::AutogradContext* ctx,
                                                  const at::Tensor& c, const at::Tensor& target,
                                                  const c10::intrusive_ptr<Ops>& ops) {
        ctx->saved_data["ops"] = c10::IValue::make_capsule(ops);
        std::vector<at::Tensor> r = ops->synthesis_sqerr(c, target);
        ctx->saved_data["y"] = r[1];
        ctx->saved_data["t"] = r[2];
        ctx->mark_non_differentiable({r[1]});
        ctx->set_materialize_grads(false);   // no zero gradient is built for y
        return {r[0], r[1]};
    }
    static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                   torch::autograd::variable_list g) {
        if (!g[0].defined()) return {at::Tensor(), at::Tensor(), at::Tensor()};
        Ops* o = ops_of(ctx);
        at::Tensor y = ctx->saved_data.at("y").toTensor();
        at::Tensor t = ctx->saved_data.at("t").toTensor();
        at::Tensor gl = g[0].to(y.options()).contiguous();
        const float scale = y.numel() > 0 ? (float)(2.0 / (double)y.numel()) : 0.f;
        at::Tensor gc = o->adj_synthesis_sqerr(y, t, scale, gl);
        at::Tensor gt;
        if (ctx->needs_input_grad(1)) gt = (y - t) * (gl * -scale);
        return {gc, gt, at::Tensor()};
    }
};

// Python handle of an Ops
struct Handle {
    c10::intrusive_ptr<Ops> ops;

    Handle(uintptr_t tables, int device, int64_t ncoef, uintptr_t an, uintptr_t syn,
           uintptr_t adj_an, uintptr_t adj_syn, uintptr_t ws_bytes, uintptr_t last_error,
           uintptr_t syn_sqerr, uintptr_t adj_syn_sqerr, pybind11::object owner, std::vector<int64_t> bins, std::vector<int64_t> lens,
           int64_t ngroups)
        : ops(c10::make_intrusive<Ops>()) {
        TORCH_CHECK(bins.size() == lens.size() && ngroups <= (int64_t)bins.size(),
                    "bad group layout");
        Ops& o = *ops;
        o.tables = reinterpret_cast<const void*>(tables);
        o.device = (c10::DeviceIndex)device;
        o.ncoef = ncoef;
        o.an = reinterpret_cast<FnSignalFirst>(an);
        o.syn = reinterpret_cast<FnCoefFirst>(syn);
        o.adj_an = reinterpret_cast<FnCoefFirst>(adj_an);
        o.adj_syn = reinterpret_cast<FnSignalFirst>(adj_syn);
        o.ws_bytes = reinterpret_cast<FnWorkspace>(ws_bytes);
        o.last_error = reinterpret_cast<FnLastError>(last_error);
        o.syn_sqerr = reinterpret_cast<FnSynSqErr>(syn_sqerr);
        o.adj_syn_sqerr = reinterpret_cast<FnAdjSynSqErr>(adj_syn_sqerr);
        o.owner = owner.release().ptr();   // the strong reference moves into Ops
        int64_t total = 0;
        for (size_t i = 0; i < bins.size(); ++i) {
            o.sizes.push_back(bins[i] * lens[i]);
            total += bins[i] * lens[i];
        }
        TORCH_CHECK(total == ncoef, "group layout does not cover the heap");
        o.bins = std::move(bins);
        o.lens = std::move(lens);
        o.ngroups = ngroups;
    }

    // the grow-only scratch for `batch` slices (shared with ctypes callers)
    at::Tensor workspace(int64_t batch) {
        size_t b;
        ops->workspace(batch, &b);
        return ops->ws;
    }

    void set_slice_len(int64_t n) {
        TORCH_CHECK_VALUE(n == 65536 || n == 32768, "slice length must be 65536 or 32768");
        ops->kN = n;
    }

    at::Tensor analysis(const at::Tensor& x) { return ops->analysis(x); }
    void analysis_planar(const at::Tensor& x, const at::Tensor& kr, const at::Tensor& ki) {
        ops->analysis_planar(x, kr, ki);
    }
    void synthesis_planar(const at::Tensor& kr, const at::Tensor& ki, const at::Tensor& y) {
        ops->synthesis_planar(kr, ki, y);
    }
    at::Tensor synthesis(const at::Tensor& c) { return ops->synthesis(c); }
    at::Tensor adj_analysis(const at::Tensor& g) { return ops->adj_analysis(g); }
    at::Tensor adj_synthesis(const at::Tensor& gy) { return ops->adj_synthesis(gy); }

    // differentiable heap <-> signal, no per-group views
    at::Tensor analysis_heap(const at::Tensor& x) { return AnalysisFn::apply(x, ops); }
    at::Tensor synthesis_heap(const at::Tensor& h) { return SynthesisFn::apply(h, ops); }
    // heap [B, ncoef] and target [B, 65536] -> (mean squared error, y)
    pybind11::tuple mse(const at::Tensor& h, const at::Tensor& target) {
        torch::autograd::variable_list r = SynthesisMSEFn::apply(h, target, ops);
        return pybind11::make_tuple(r[0], r[1]);
    }

    // TrainableCQT.fwd: x [..., 65536] -> (blocks [..., b, M], side [..., 1, M])
    pybind11::tuple fwd(const at::Tensor& x) {
        Ops& o = *ops;
        TORCH_CHECK(x.dim() >= 1 && x.size(-1) == ops->kN, "x must be [..., ", ops->kN, "]");
        std::vector<int64_t> lead(x.sizes().begin(), x.sizes().end() - 1);
        int64_t B = 1;   // explicit: reshape cannot infer -1 for an empty batch
        for (int64_t d : lead) B *= d;
        // a [B, 65536] input goes in as it is: a no-op reshape would still
        // add a view node to the autograd graph
        at::Tensor h = AnalysisFn::apply(x.dim() == 2 ? x : x.reshape({B, ops->kN}), ops);
        std::vector<at::Tensor> parts = h.split_with_sizes(o.sizes, 1);
        pybind11::list blocks, side;
        o.last_v.clear();
        std::vector<int64_t> shape(lead);
        shape.push_back(0);
        shape.push_back(0);
        for (size_t i = 0; i < parts.size(); ++i) {
            shape[shape.size() - 2] = o.bins[i];
            shape[shape.size() - 1] = o.lens[i];
            at::Tensor v = parts[i].view(shape);
            o.last_v.emplace_back(v.getIntrusivePtr());
            if ((int64_t)i < o.ngroups) blocks.append(v);
            else side.append(v);
        }
        o.last_h = c10::weak_intrusive_ptr<c10::TensorImpl, c10::UndefinedTensorImpl>(
            h.getIntrusivePtr());
        return pybind11::make_tuple(blocks, side);
    }

    // the heap behind (blocks, side) when they are the untouched views the last
    // fwd returned (same tensor objects, the heap still alive), else None
    pybind11::object last_heap(const std::vector<at::Tensor>& all) {
        Ops& o = *ops;
        if (all.size() != o.last_v.size() || o.last_h.expired()) return pybind11::none();
        for (size_t i = 0; i < all.size(); ++i)
            if (o.last_v[i].expired() ||
                all[i].unsafeGetTensorImpl() != o.last_v[i]._unsafe_get_target())
                return pybind11::none();
        auto hp = o.last_h.lock();
        if (!hp) return pybind11::none();
        return pybind11::cast(at::Tensor(std::move(hp)));
    }

    // TrainableCQT.mse_loss in one call when (blocks, side) are the untouched
    // views of the last fwd: the target [lead..., 65536] is checked and
    // flattened here; (loss, y [lead..., 65536]) or None (the caller takes the
    // general path)
    pybind11::object mse_views(const std::vector<at::Tensor>& all, const at::Tensor& target) {
        pybind11::object h = last_heap(all);
        if (h.is_none()) return pybind11::none();
        at::Tensor heap = h.cast<at::Tensor>();
        const int64_t B = heap.size(0);
        std::vector<int64_t> lead(all[0].sizes().begin(), all[0].sizes().end() - 2);
        std::vector<int64_t> want(lead);
        want.push_back(ops->kN);
        TORCH_CHECK_VALUE(target.defined() && target.sizes().vec() == want, "target must be ",
                          c10::IntArrayRef(want), ", got ",
                          target.defined() ? target.sizes() : c10::IntArrayRef());
        torch::autograd::variable_list r =
            SynthesisMSEFn::apply(heap, target.dim() == 2 ? target : target.reshape({B, ops->kN}), ops);
        at::Tensor y = lead.size() == 1 ? r[1] : r[1].reshape(want);
        return pybind11::make_tuple(r[0], y);
    }
};

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "torch fast path of the flash_cqt_b200 C ABI";
    pybind11::class_<Handle>(m, "Handle")
        .def(pybind11::init<uintptr_t, int, int64_t, uintptr_t, uintptr_t, uintptr_t, uintptr_t,
                            uintptr_t, uintptr_t, uintptr_t, uintptr_t, pybind11::object,
                            std::vector<int64_t>, std::vector<int64_t>, int64_t>())
        .def("workspace", &Handle::workspace)
        .def("set_slice_len", &Handle::set_slice_len)
        .def("analysis", &Handle::analysis)
        .def("analysis_planar", &Handle::analysis_planar)
        .def("synthesis_planar", &Handle::synthesis_planar)
        .def("synthesis", &Handle::synthesis)
        .def("adj_analysis", &Handle::adj_analysis)
        .def("adj_synthesis", &Handle::adj_synthesis)
        .def("analysis_heap", &Handle::analysis_heap)
        .def("synthesis_heap", &Handle::synthesis_heap)
        .def("mse", &Handle::mse)
        .def("mse_views", &Handle::mse_views)
        .def("fwd", &Handle::fwd)
        .def("last_heap", &Handle::last_heap);
}
