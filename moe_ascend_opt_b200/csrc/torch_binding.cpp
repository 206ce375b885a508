// PyTorch binding of the engine: the reference's `nanovllm` operator surface
// (Int8-gemm/nanovllm_ops.cpp:349-431) registered for the CUDA dispatch key,
// implemented on top of the C ABI of include/moe_b200.h.
//
//   torch.classes.nanovllm.MoEInfer(E, H, I, quant_type)        nanovllm_ops.cpp:350-353
//     .quantize_and_store_expert(e, proj, w)                    :354-365 (Q8_0 only)
//     .store_quantized_repack(gate_up_qs, gate_up_d, down_qs, down_d)  :366-371
//     .get_last_run_time_ms() / get_quant_type() / get_num_experts() /
//      get_hidden_size() / get_intermediate_size()              :372-391
//     new: store_awq(...), set_expert_parallel(rank, size), set_group_size(g),
//          p2p_mailbox / p2p_connect / p2p_covers / p2p_enable (peer-memory combine),
//          reserve(T, K), export_expert(e, which), device_error()
//   torch.ops.nanovllm.moe_forward(hidden, topk_ids, topk_w, moe)          :402
//   torch.ops.nanovllm.moe_forward_npu_stream(...)   same schema, CUDA stream :405
//   torch.ops.nanovllm.moe_forward_npu_graph_out(..., ctx, out)            :406
//   torch.classes.nanovllm.MoEGraphContext(moe, num_tokens, top_k, dtype)  :398-399
//   torch.classes.nanovllm.NpuCallbackManager(stream_ptr, device_id)       :395-396 (no-op)
//   new: moe_forward_partial, moe_dense_forward, moe_route, moe_route_gemm, moe_route_permute,
//        quantize_rows_q8_0
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/custom_class.h>
#include <torch/library.h>
#include <torch/torch.h>

#include <algorithm>
#include <string>

#include "../../include/moe_b200.h"

namespace {

void check_rc(int rc, const char* what) {
    TORCH_CHECK(rc == MOE_OK, what, " failed: ", moe_last_error());
}

void* cur_stream(int device) { return (void*)at::cuda::getCurrentCUDAStream(device).stream(); }

int32_t dtype_code(at::ScalarType t) {
    if (t == at::kHalf) return MOE_F16;
    if (t == at::kBFloat16) return MOE_BF16;
    if (t == at::kFloat) return MOE_F32;
    TORCH_CHECK(false, "unsupported dtype ", t);
}

struct MoEInferHandle : torch::CustomClassHolder {
    int64_t E, H, I;
    int64_t quant_type;
    int64_t group_size = 128;
    int64_t ep_rank = 0, ep_size = 1;
    std::vector<int64_t> placement;  // global ids of the experts held here, in local order (empty: contiguous block)
    std::vector<int64_t> replicas;   // hot experts held by every rank (a subset of placement)
    moe_engine* eng = nullptr;
    int device = -1;

    MoEInferHandle(int64_t E_, int64_t H_, int64_t I_, int64_t qt) : E(E_), H(H_), I(I_), quant_type(qt) {
        TORCH_CHECK(qt == MOE_Q8_0 || qt == MOE_Q4_0 || qt == MOE_AWQ, "quant_type must be 0 (Q8_0), 1 (Q4_0) or 2 (AWQ)");
        TORCH_CHECK(H % 32 == 0, "hidden_size must be multiple of 32");
        TORCH_CHECK(I % 32 == 0, "intermediate_size must be multiple of 32");
    }
    ~MoEInferHandle() override {
        if (eng) moe_engine_destroy(eng);
    }

    int64_t local_experts() const { return placement.empty() ? E / ep_size : (int64_t)placement.size(); }
    int64_t expert_offset() const { return placement.empty() ? ep_rank * local_experts() : 0; }
    int64_t local_of(int64_t e) const {  // -1: another rank's expert
        if (placement.empty()) return (e >= expert_offset() && e < expert_offset() + local_experts()) ? e - expert_offset() : -1;
        for (size_t l = 0; l < placement.size(); ++l)
            if (placement[l] == e) return (int64_t)l;
        return -1;
    }
    void set_expert_placement(const std::vector<int64_t>& experts) {
        TORCH_CHECK(!eng, "set_expert_placement must precede weight loading");
        TORCH_CHECK(!experts.empty(), "empty placement");
        std::vector<char> seen(E, 0);
        for (int64_t e : experts) {
            TORCH_CHECK(e >= 0 && e < E && !seen[e], "placement: expert ids must be distinct and in [0, E)");
            seen[e] = 1;
        }
        placement = experts;
    }

    void set_expert_replicas(const std::vector<int64_t>& hot) {
        TORCH_CHECK(!eng, "set_expert_replicas must precede weight loading");
        TORCH_CHECK(!placement.empty(), "set_expert_placement (including the replicated experts) first");
        for (int64_t e : hot)
            TORCH_CHECK(std::find(placement.begin(), placement.end(), e) != placement.end(),
                        "replicated expert ", e, " is not in this rank's placement");
        replicas = hot;
    }

    void set_expert_parallel(int64_t rank, int64_t size) {
        TORCH_CHECK(!eng, "set_expert_parallel must precede weight loading");
        TORCH_CHECK(size >= 1 && rank >= 0 && rank < size, "bad expert-parallel config");
        ep_rank = rank;
        ep_size = size;
    }
    void set_group_size(int64_t g) {
        TORCH_CHECK(!eng, "set_group_size must precede weight loading");
        group_size = g;
    }

    void ensure_engine() {
        if (eng) return;
        TORCH_CHECK(!placement.empty() || E % ep_size == 0,
                    "bad expert-parallel config: contiguous expert blocks need E divisible by the world size");
        device = at::cuda::current_device();
        moe_config cfg{};
        cfg.num_experts = local_experts();
        cfg.hidden_size = H;
        cfg.intermediate_size = I;
        cfg.quant_type = (int32_t)quant_type;
        cfg.group_size = (int32_t)group_size;
        cfg.device = device;
        cfg.expert_offset = (int32_t)expert_offset();
        check_rc(moe_engine_create(&cfg, &eng), "moe_engine_create");
        if (!placement.empty()) {
            std::vector<int32_t> m(E, -1);
            for (size_t l = 0; l < placement.size(); ++l) m[placement[l]] = (int32_t)l;
            for (int64_t e : replicas) m[e] |= MOE_REPLICATED;
            check_rc(moe_engine_set_replica_split(eng, (int32_t)ep_rank, (int32_t)ep_size), "set_expert_replicas");
            check_rc(moe_engine_set_expert_map(eng, m.data(), E), "set_expert_placement");
        }
    }

    // slice the local experts of a full [E, ...] tensor and make it contiguous
    at::Tensor local(const at::Tensor& t) const {
        TORCH_CHECK(t.dim() == 3 && t.size(0) == E, "E mismatch");
        if (!placement.empty()) {
            auto idx = at::tensor(placement, at::TensorOptions().dtype(at::kLong)).to(t.device());
            return t.index_select(0, idx).contiguous();
        }
        if (ep_size == 1) return t.contiguous();
        return t.narrow(0, expert_offset(), local_experts()).contiguous();
    }

    void store_quantized_repack(const at::Tensor& gu_qs, const at::Tensor& gu_d, const at::Tensor& dn_qs,
                                const at::Tensor& dn_d) {
        TORCH_CHECK(quant_type != MOE_AWQ, "AWQ handle: use store_awq");
        TORCH_CHECK(gu_d.scalar_type() == at::kHalf || gu_d.scalar_type() == at::kBFloat16,
                    "gate_up_d must be float16 or bfloat16");
        TORCH_CHECK(dn_d.scalar_type() == gu_d.scalar_type(), "gate_up_d and down_proj_d must have the same dtype");
        TORCH_CHECK(gu_qs.dim() == 3, "gate_up_qs must be [E,2I,H]");
        TORCH_CHECK(dn_qs.dim() == 3, "down_proj_qs must be [E,H,I]");
        if (quant_type == MOE_Q4_0) {
            TORCH_CHECK(gu_qs.scalar_type() == at::kInt || gu_qs.scalar_type() == at::kUInt32,
                        "Q4_0 gate_up_qs must be int32 (uint32 storage)");
            TORCH_CHECK(dn_qs.scalar_type() == at::kInt || dn_qs.scalar_type() == at::kUInt32,
                        "Q4_0 down_proj_qs must be int32 (uint32 storage)");
            TORCH_CHECK(gu_qs.size(1) == 2 * I && gu_qs.size(2) == H / 8 && dn_qs.size(1) == H && dn_qs.size(2) == I / 8,
                        "Q4_0 weight shapes must be [E,2I,H/8] and [E,H,I/8]");
        } else {
            TORCH_CHECK(gu_qs.scalar_type() == at::kChar, "Q8_0 gate_up_qs must be int8");
            TORCH_CHECK(dn_qs.scalar_type() == at::kChar, "Q8_0 down_proj_qs must be int8");
            TORCH_CHECK(gu_qs.size(1) == 2 * I && gu_qs.size(2) == H && dn_qs.size(1) == H && dn_qs.size(2) == I,
                        "Q8_0 weight shapes must be [E,2I,H] and [E,H,I]");
        }
        TORCH_CHECK(gu_d.dim() == 3 && gu_d.size(1) == 2 * I && gu_d.size(2) == H / 32, "gate_up_d must be [E,2I,H/32]");
        TORCH_CHECK(dn_d.dim() == 3 && dn_d.size(1) == H && dn_d.size(2) == I / 32, "down_proj_d must be [E,H,I/32]");
        ensure_engine();
        c10::cuda::CUDAGuard g(device);
        auto a = local(gu_qs), b = local(gu_d), c = local(dn_qs), d = local(dn_d);
        const bool on_dev = a.is_cuda();
        TORCH_CHECK(b.is_cuda() == on_dev && c.is_cuda() == on_dev && d.is_cuda() == on_dev,
                    "weights must all be on the same device type");
        check_rc(moe_engine_load_quantized(eng, a.data_ptr(), b.data_ptr(), c.data_ptr(), d.data_ptr(),
                                           dtype_code(b.scalar_type()), on_dev ? 1 : 0, cur_stream(device)),
                 "store_quantized_repack");
    }

    void quantize_and_store_expert(int64_t e, const std::string& proj, const at::Tensor& w) {
        TORCH_CHECK(quant_type != MOE_Q4_0,
                    "Q4_0 does not support online quantization. Use store_quantized_repack() with pre-quantized weights.");
        TORCH_CHECK(quant_type == MOE_Q8_0, "online quantization is Q8_0 only");
        TORCH_CHECK(w.dim() == 2, "Weight must be 2D");
        TORCH_CHECK(w.scalar_type() == at::kFloat || w.scalar_type() == at::kHalf || w.scalar_type() == at::kBFloat16,
                    "Weight must be float32, float16 or bfloat16 for quantize_weight_only");
        int32_t p;
        if (proj == "gate_proj") {
            p = 0;
        } else if (proj == "up_proj") {
            p = 1;
        } else if (proj == "down_proj") {
            p = 2;
        } else {
            TORCH_CHECK(false, "Unknown proj_name: ", proj);
        }
        if (p < 2) {
            TORCH_CHECK(w.size(0) == I && w.size(1) == H, "gate/up weight must be [I,H]");
        } else {
            TORCH_CHECK(w.size(0) == H && w.size(1) == I, "down weight must be [H,I]");
        }
        TORCH_CHECK(e >= 0 && e < E, "expert index out of range");
        const int64_t le = local_of(e);
        if (le < 0) return;  // another rank's expert
        ensure_engine();
        c10::cuda::CUDAGuard g(device);
        auto wc = w.contiguous();
        check_rc(moe_engine_quantize_store_expert(eng, le, p, wc.data_ptr(), dtype_code(wc.scalar_type()),
                                                  wc.is_cuda() ? 1 : 0, cur_stream(device)),
                 "quantize_and_store_expert");
    }

    void store_awq(const at::Tensor& w13_qw, const at::Tensor& w13_sc, const at::Tensor& w13_qz,
                   const at::Tensor& w2_qw, const at::Tensor& w2_sc, const at::Tensor& w2_qz) {
        TORCH_CHECK(quant_type == MOE_AWQ, "store_awq needs quant_type 2 (AWQ)");
        const int64_t G = group_size;
        TORCH_CHECK(w13_qw.scalar_type() == at::kInt && w13_qz.scalar_type() == at::kInt &&
                        w2_qw.scalar_type() == at::kInt && w2_qz.scalar_type() == at::kInt,
                    "AWQ qweight / qzeros must be int32");
        TORCH_CHECK(w13_sc.scalar_type() == at::kBFloat16 && w2_sc.scalar_type() == at::kBFloat16,
                    "AWQ scales must be bfloat16");
        TORCH_CHECK(w13_qw.size(1) == H && w13_qw.size(2) == 2 * I / 8, "w13_qweight must be [E,H,2I/8]");
        TORCH_CHECK(w13_sc.size(1) == H / G && w13_sc.size(2) == 2 * I, "w13_scales must be [E,H/G,2I]");
        TORCH_CHECK(w13_qz.size(1) == H / G && w13_qz.size(2) == 2 * I / 8, "w13_qzeros must be [E,H/G,2I/8]");
        TORCH_CHECK(w2_qw.size(1) == I && w2_qw.size(2) == H / 8, "w2_qweight must be [E,I,H/8]");
        TORCH_CHECK(w2_sc.size(1) == I / G && w2_sc.size(2) == H, "w2_scales must be [E,I/G,H]");
        TORCH_CHECK(w2_qz.size(1) == I / G && w2_qz.size(2) == H / 8, "w2_qzeros must be [E,I/G,H/8]");
        ensure_engine();
        c10::cuda::CUDAGuard g(device);
        at::Tensor t[6] = {local(w13_qw), local(w13_sc), local(w13_qz), local(w2_qw), local(w2_sc), local(w2_qz)};
        const bool on_dev = t[0].is_cuda();
        for (auto& x : t) TORCH_CHECK(x.is_cuda() == on_dev, "weights must all be on the same device type");
        check_rc(moe_engine_load_awq(eng, t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), t[3].data_ptr(),
                                     t[4].data_ptr(), t[5].data_ptr(), on_dev ? 1 : 0, cur_stream(device)),
                 "store_awq");
    }

    void forward_into(const at::Tensor& hidden, const at::Tensor& ids, const at::Tensor& w, at::Tensor& out) {
        TORCH_CHECK(eng, "no weights loaded");
        TORCH_CHECK(hidden.is_cuda() && ids.is_cuda() && w.is_cuda() && out.is_cuda(), "tensors must be CUDA tensors");
        TORCH_CHECK(hidden.get_device() == device, "hidden must be on the engine's device");
        TORCH_CHECK(hidden.dim() == 2 && hidden.size(1) == H, "hidden must be [T, H]");
        TORCH_CHECK(hidden.scalar_type() == at::kHalf || hidden.scalar_type() == at::kBFloat16,
                    "hidden must be float16 or bfloat16");
        TORCH_CHECK(ids.scalar_type() == at::kInt && ids.dim() == 2 && ids.size(0) == hidden.size(0),
                    "topk_ids must be int32 [T, K]");
        TORCH_CHECK(w.scalar_type() == at::kFloat && w.sizes() == ids.sizes(), "topk_w must be float32 [T, K]");
        TORCH_CHECK(hidden.is_contiguous() && ids.is_contiguous() && w.is_contiguous() && out.is_contiguous(),
                    "tensors must be contiguous");
        TORCH_CHECK(out.sizes() == hidden.sizes(), "out must be [T, H]");
        c10::cuda::CUDAGuard g(device);
        check_rc(moe_engine_forward(eng, hidden.data_ptr(), out.data_ptr(), ids.data_ptr<int32_t>(), w.data_ptr<float>(),
                                    hidden.size(0), ids.size(1), dtype_code(hidden.scalar_type()),
                                    dtype_code(out.scalar_type()), cur_stream(device)),
                 "moe_forward");
    }

    // expert-parallel combine over peer memory (include/moe_b200.h, moe_engine_p2p_*)
    at::Tensor p2p_mailbox(int64_t world, int64_t max_tokens) {
        TORCH_CHECK(eng, "no weights loaded");
        TORCH_CHECK(world == ep_size, "world must equal the expert-parallel size");
        c10::cuda::CUDAGuard g(device);
        auto h = at::zeros({64}, at::TensorOptions().dtype(at::kByte));
        check_rc(moe_engine_p2p_mailbox(eng, (int32_t)world, max_tokens, h.data_ptr()), "p2p_mailbox");
        return h;
    }
    void p2p_connect(const at::Tensor& handles) {
        TORCH_CHECK(eng, "no weights loaded");
        auto h = handles.to(at::kCPU).contiguous();
        TORCH_CHECK(h.scalar_type() == at::kByte && h.numel() == ep_size * 64, "handles must be uint8 [world, 64]");
        c10::cuda::CUDAGuard g(device);
        check_rc(moe_engine_p2p_connect(eng, (int32_t)ep_rank, (int32_t)ep_size, h.data_ptr()), "p2p_connect");
    }
    bool p2p_covers(int64_t T) { return eng && moe_engine_p2p_covers(eng, T); }
    void p2p_enable(bool on) {
        TORCH_CHECK(eng, "no weights loaded");
        check_rc(moe_engine_p2p_enable(eng, on ? 1 : 0), "p2p_enable");
    }

    double last_ms() {
        if (!eng) return 0.0;
        double ms = 0.0;
        check_rc(moe_engine_last_time_ms(eng, &ms), "get_last_run_time_ms");
        return ms;
    }
};

struct MoEGraphContext : torch::CustomClassHolder {
    int64_t num_tokens, top_k, dtype_int;
    MoEGraphContext(const c10::intrusive_ptr<MoEInferHandle>& moe, int64_t T, int64_t K, int64_t dt)
        : num_tokens(T), top_k(K), dtype_int(dt) {
        TORCH_CHECK(dt == 0 || dt == 1, "dtype_int must be 0 (float16) or 1 (bfloat16)");
        TORCH_CHECK(moe->eng, "load weights before creating a MoEGraphContext");
        check_rc(moe_engine_reserve(moe->eng, T, K), "MoEGraphContext reserve");
    }
};

struct NpuCallbackManager : torch::CustomClassHolder {
    // The reference needs a host callback thread per NPU stream; CUDA execution is
    // stream ordered on the device, so this class only keeps imports working.
    NpuCallbackManager(int64_t, int64_t) {}
};

at::Tensor moe_forward(const at::Tensor& hidden, const at::Tensor& ids, const at::Tensor& w,
                       const c10::intrusive_ptr<MoEInferHandle>& moe) {
    auto out = at::empty_like(hidden);
    moe->forward_into(hidden, ids, w, out);
    return out;
}

at::Tensor moe_dense_forward(const at::Tensor& hidden, int64_t expert, const c10::intrusive_ptr<MoEInferHandle>& moe) {
    TORCH_CHECK(moe->eng, "no weights loaded");
    TORCH_CHECK(hidden.is_cuda() && hidden.dim() == 2 && hidden.size(1) == moe->H && hidden.is_contiguous(),
                "hidden must be a contiguous CUDA [T, H] tensor");
    TORCH_CHECK(hidden.scalar_type() == at::kHalf || hidden.scalar_type() == at::kBFloat16,
                "hidden must be float16 or bfloat16");
    c10::cuda::CUDAGuard g(moe->device);
    auto out = at::empty_like(hidden);
    const int64_t le = moe->local_of(expert);
    TORCH_CHECK(le >= 0, "expert ", expert, " is not held by this rank");
    check_rc(moe_engine_forward_dense(moe->eng, le, hidden.data_ptr(), out.data_ptr(), hidden.size(0),
                                      dtype_code(hidden.scalar_type()), dtype_code(out.scalar_type()),
                                      cur_stream(moe->device)),
             "moe_dense_forward");
    return out;
}

at::Tensor moe_forward_partial(const at::Tensor& hidden, const at::Tensor& ids, const at::Tensor& w,
                               const c10::intrusive_ptr<MoEInferHandle>& moe) {
    auto out = at::empty(hidden.sizes(), hidden.options().dtype(at::kFloat));
    moe->forward_into(hidden, ids, w, out);
    return out;
}

void moe_forward_graph_out(const at::Tensor& hidden, const at::Tensor& ids, const at::Tensor& w,
                           const c10::intrusive_ptr<MoEInferHandle>& moe, const c10::intrusive_ptr<MoEGraphContext>& ctx,
                           at::Tensor out) {
    TORCH_CHECK(hidden.size(0) <= ctx->num_tokens && ids.size(1) <= ctx->top_k, "input exceeds the MoEGraphContext");
    moe->forward_into(hidden, ids, w, out);
}

std::tuple<at::Tensor, at::Tensor> moe_route(const at::Tensor& logits, int64_t K, bool renormalize) {
    TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.dim() == 2, "logits must be CUDA fp32 [T,E]");
    auto l = logits.contiguous();
    c10::cuda::CUDAGuard g(l.get_device());
    auto ids = at::empty({l.size(0), K}, l.options().dtype(at::kInt));
    auto w = at::empty({l.size(0), K}, l.options());
    check_rc(moe_route_topk(l.data_ptr<float>(), l.size(0), l.size(1), K, renormalize ? 1 : 0, ids.data_ptr<int32_t>(),
                            w.data_ptr<float>(), cur_stream(l.get_device())),
             "moe_route");
    return {ids, w};
}

std::tuple<at::Tensor, at::Tensor> moe_route_gemm(const at::Tensor& hidden, const at::Tensor& weight, int64_t K,
                                                  bool renormalize) {
    TORCH_CHECK(hidden.is_cuda() && weight.is_cuda() && hidden.dim() == 2 && weight.dim() == 2 &&
                    weight.size(1) == hidden.size(1),
                "hidden [T,H] and router weight [E,H] must be CUDA tensors");
    auto x = hidden.contiguous();
    auto w = weight.contiguous();
    c10::cuda::CUDAGuard g(x.get_device());
    auto ids = at::empty({x.size(0), K}, x.options().dtype(at::kInt));
    auto tw = at::empty({x.size(0), K}, x.options().dtype(at::kFloat));
    check_rc(moe_route_gemm_topk(x.data_ptr(), dtype_code(x.scalar_type()), w.data_ptr(), dtype_code(w.scalar_type()),
                                 x.size(0), x.size(1), w.size(0), K, renormalize ? 1 : 0, ids.data_ptr<int32_t>(),
                                 tw.data_ptr<float>(), nullptr, cur_stream(x.get_device())),
             "moe_route_gemm");
    return {ids, tw};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> route_permute(const at::Tensor& ids, int64_t E) {
    TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kInt && ids.dim() == 2, "ids must be CUDA int32 [T,K]");
    auto x = ids.contiguous();
    c10::cuda::CUDAGuard g(x.get_device());
    const int64_t TK = x.numel();
    auto o = x.options();
    auto counts = at::empty({E}, o), starts = at::empty({E + 1}, o);
    auto tmap = at::full({std::max<int64_t>(TK, 1), 2}, -1, o), smap = at::empty({x.size(0), x.size(1)}, o);
    check_rc(moe_route_permute(x.data_ptr<int32_t>(), x.size(0), x.size(1), E, counts.data_ptr<int32_t>(),
                               starts.data_ptr<int32_t>(), tmap.data_ptr<int32_t>(), smap.data_ptr<int32_t>(),
                               cur_stream(x.get_device())),
             "moe_route_permute");
    return {counts, starts, tmap, smap};
}

std::tuple<at::Tensor, at::Tensor> quantize_rows(const at::Tensor& x) {
    TORCH_CHECK(x.is_cuda() && x.dim() == 2, "x must be a CUDA [rows, cols] tensor");
    auto c = x.contiguous();
    c10::cuda::CUDAGuard g(c.get_device());
    auto qs = at::empty(c.sizes(), c.options().dtype(at::kChar));
    auto d = at::empty({c.size(0), c.size(1) / 32}, c.options().dtype(at::kFloat));
    check_rc(moe_quantize_rows_q8_0(c.data_ptr(), dtype_code(c.scalar_type()), c.size(0), c.size(1),
                                    qs.data_ptr<int8_t>(), d.data_ptr<float>(), cur_stream(c.get_device())),
             "quantize_rows_q8_0");
    return {qs, d};
}

}  // namespace

TORCH_LIBRARY_FRAGMENT(nanovllm, m) {
    m.class_<MoEInferHandle>("MoEInfer")
        .def(torch::init<int64_t, int64_t, int64_t, int64_t>())
        .def("quantize_and_store_expert", &MoEInferHandle::quantize_and_store_expert)
        .def("store_quantized_repack", &MoEInferHandle::store_quantized_repack)
        .def("store_awq", &MoEInferHandle::store_awq)
        .def("set_expert_parallel", &MoEInferHandle::set_expert_parallel)
        .def("set_expert_placement", &MoEInferHandle::set_expert_placement)
        .def("set_expert_replicas", &MoEInferHandle::set_expert_replicas)
        .def("engine_handle",  // the moe_engine* behind this handle, for direct C-ABI calls (include/moe_b200.h)
             [](const c10::intrusive_ptr<MoEInferHandle>& s) -> int64_t {
                 TORCH_CHECK(s->eng, "no weights loaded");
                 return (int64_t)reinterpret_cast<intptr_t>(s->eng);
             })
        .def("set_group_size", &MoEInferHandle::set_group_size)
        .def("save",  // the device-resident packed layouts to a file (include/moe_b200.h, moe_engine_save)
             [](const c10::intrusive_ptr<MoEInferHandle>& s, const std::string& path) {
                 TORCH_CHECK(s->eng, "no weights loaded");
                 check_rc(moe_engine_save(s->eng, path.c_str()), "save");
             })
        .def("load_file",  // fill the engine from such a file, no repacking
             [](const c10::intrusive_ptr<MoEInferHandle>& s, const std::string& path) {
                 s->ensure_engine();
                 check_rc(moe_engine_load_file(s->eng, path.c_str()), "load_file");
             })
        .def("p2p_mailbox", &MoEInferHandle::p2p_mailbox)
        .def("p2p_connect", &MoEInferHandle::p2p_connect)
        .def("p2p_covers", &MoEInferHandle::p2p_covers)
        .def("p2p_enable", &MoEInferHandle::p2p_enable)
        .def("get_last_run_time_ms", [](const c10::intrusive_ptr<MoEInferHandle>& s) { return s->last_ms(); })
        .def("get_quant_type",
             [](const c10::intrusive_ptr<MoEInferHandle>& s) -> std::string {
                 return s->quant_type == MOE_Q4_0 ? "Q4_0" : (s->quant_type == MOE_AWQ ? "AWQ" : "Q8_0");
             })
        .def("get_num_experts", [](const c10::intrusive_ptr<MoEInferHandle>& s) { return s->E; })
        .def("get_hidden_size", [](const c10::intrusive_ptr<MoEInferHandle>& s) { return s->H; })
        .def("get_intermediate_size", [](const c10::intrusive_ptr<MoEInferHandle>& s) { return s->I; })
        .def("reserve",
             [](const c10::intrusive_ptr<MoEInferHandle>& s, int64_t T, int64_t K) {
                 TORCH_CHECK(s->eng, "no weights loaded");
                 check_rc(moe_engine_reserve(s->eng, T, K), "reserve");
             })
        .def("device_error",
             [](const c10::intrusive_ptr<MoEInferHandle>& s) -> int64_t {
                 if (!s->eng) return 0;
                 int32_t c = 0;
                 check_rc(moe_engine_device_error(s->eng, &c), "device_error");
                 return c;
             })
        .def("export_expert", [](const c10::intrusive_ptr<MoEInferHandle>& s, int64_t e, int64_t which) {
            TORCH_CHECK(s->eng, "no weights loaded");
            const bool q4 = s->quant_type == MOE_Q4_0;
            const int64_t rows = which == 0 ? 2 * s->I : s->H, cols = which == 0 ? s->H : s->I;
            at::Tensor qs = q4 ? at::empty({rows, cols / 8}, at::kInt) : at::empty({rows, cols}, at::kChar);
            at::Tensor d = at::empty({rows, cols / 32}, at::kShort);
            check_rc(moe_engine_export_expert(s->eng, e, (int32_t)which, qs.data_ptr(), d.data_ptr()), "export_expert");
            return std::vector<at::Tensor>{qs, d};
        });
    m.class_<MoEGraphContext>("MoEGraphContext")
        .def(torch::init<const c10::intrusive_ptr<MoEInferHandle>&, int64_t, int64_t, int64_t>());
    m.class_<NpuCallbackManager>("NpuCallbackManager").def(torch::init<int64_t, int64_t>());

    m.def("moe_forward(Tensor hidden, Tensor topk_ids, Tensor topk_w, __torch__.torch.classes.nanovllm.MoEInfer moe) -> Tensor");
    m.def("moe_forward_npu_stream(Tensor hidden, Tensor topk_ids, Tensor topk_w, __torch__.torch.classes.nanovllm.MoEInfer moe) -> Tensor");
    m.def("moe_forward_npu_graph_out(Tensor hidden, Tensor topk_ids, Tensor topk_w, __torch__.torch.classes.nanovllm.MoEInfer moe, __torch__.torch.classes.nanovllm.MoEGraphContext ctx, Tensor(a!) out) -> ()");
    m.def("moe_forward_partial(Tensor hidden, Tensor topk_ids, Tensor topk_w, __torch__.torch.classes.nanovllm.MoEInfer moe) -> Tensor");
    m.def("moe_route(Tensor logits, int top_k, bool renormalize) -> (Tensor, Tensor)");
    m.def("moe_dense_forward(Tensor hidden, int expert, __torch__.torch.classes.nanovllm.MoEInfer moe) -> Tensor");
    m.def("moe_route_gemm(Tensor hidden, Tensor router_weight, int top_k, bool renormalize) -> (Tensor, Tensor)");
    m.def("moe_route_permute(Tensor topk_ids, int num_experts) -> (Tensor, Tensor, Tensor, Tensor)");
    m.def("quantize_rows_q8_0(Tensor x) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(nanovllm, CUDA, m) {
    m.impl("moe_forward", &moe_forward);
    m.impl("moe_forward_npu_stream", &moe_forward);
    m.impl("moe_forward_npu_graph_out", &moe_forward_graph_out);
    m.impl("moe_forward_partial", &moe_forward_partial);
    m.impl("moe_route", &moe_route);
    m.impl("moe_dense_forward", &moe_dense_forward);
    m.impl("moe_route_gemm", &moe_route_gemm);
    m.impl("moe_route_permute", &route_permute);
    m.impl("quantize_rows_q8_0", &quantize_rows);
}
