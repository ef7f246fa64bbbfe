// aero_cuda_moe_open_gguf: read one MoE layer out of a GGUF file and open it.
//
// Tensor names and metadata keys follow the reference's qwen35moe reading
// (engine/moe.py:5-12, engine/model.py:193-224): expert_count and
// expert_used_count come from "<arch>.expert_count" / "<arch>.expert_used_count"
// (falling back to the expert axis of ffn_gate_exps), ffn_len from the tensor
// shape, norm_topk_prob is 1, the shared expert is present when
// ffn_gate_shexp.weight is.
#include <cuda_runtime.h>

#include <cstdio>
#include <string>
#include <utility>
#include <vector>

#include "../../include/aero_cuda_moe.h"
#include "gguf_loader.h"
#include "internal.h"

namespace {

void put_err(char* err, int errlen, const std::string& s) {
    if (err && errlen > 0) std::snprintf(err, (size_t)errlen, "%s", s.c_str());
}

// f32 copy of a small F32 / F16 tensor on the device (router, shared gate).
float* small_f32(const aero::GgufFile& f, const aero::GgufTensor& t, int device, std::vector<std::pair<void*, size_t>>& tmp,
                 std::string* why) {
    if (t.type != 0 && t.type != 1) {
        *why = t.name + ": only F32 or F16 router tensors are supported";
        return nullptr;
    }
    cudaSetDevice(device);
    void* dst = nullptr;
    if (aero::guarded_malloc(&dst, (size_t)t.n_values * 4, aero::kScratch) != cudaSuccess) {
        cudaGetLastError();
        *why = t.name + ": staging allocation refused";
        return nullptr;
    }
    tmp.push_back({dst, (size_t)t.n_values * 4});
    if (t.type == 0) {
        if (cudaMemcpy(dst, f.data(t), (size_t)t.n_values * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            *why = t.name + ": upload failed";
            return nullptr;
        }
        return (float*)dst;
    }
    void* h16 = nullptr;
    if (aero::guarded_malloc(&h16, (size_t)t.n_values * 2, aero::kScratch) != cudaSuccess) {
        cudaGetLastError();
        *why = t.name + ": staging allocation refused";
        return nullptr;
    }
    tmp.push_back({h16, (size_t)t.n_values * 2});
    if (cudaMemcpy(h16, f.data(t), (size_t)t.n_values * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        aero::launch_f16_to_f32((const uint16_t*)h16, t.n_values, (float*)dst, 0) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        *why = t.name + ": f16 conversion failed";
        return nullptr;
    }
    return (float*)dst;
}

// One MoE layer's tensors in an open GGUF file, with their shapes checked.
struct LayerTensors {
    const aero::GgufTensor *gate = nullptr, *up = nullptr, *down = nullptr, *router = nullptr;
    const aero::GgufTensor *sh_inp = nullptr, *sh_gate = nullptr, *sh_up = nullptr, *sh_down = nullptr;
    int64_t E = 0, F = 0, d = 0, n_used = -1, Fs = 0;
};

bool find_layer(const aero::GgufFile& f, int layer, LayerTensors* L, std::string* why) {
    const std::string p = "blk." + std::to_string(layer) + ".";
    L->gate = f.find(p + "ffn_gate_exps.weight");
    L->up = f.find(p + "ffn_up_exps.weight");
    L->down = f.find(p + "ffn_down_exps.weight");
    L->router = f.find(p + "ffn_gate_inp.weight");
    const aero::GgufTensor *tg = L->gate, *tu = L->up, *td = L->down;
    if (!tg || !tu || !td) {
        *why = p + "ffn_{gate,up,down}_exps.weight missing: not a MoE layer";
        return false;
    }
    if (tg->dims.size() != 3 || tu->dims.size() != 3 || td->dims.size() != 3) {
        *why = p + "expert tensors must be 3-D (n_expert, out, in)";
        return false;
    }
    L->E = tg->shape(0);
    L->F = tg->shape(1);
    L->d = tg->shape(2);
    if (tu->shape(0) != L->E || tu->shape(1) != L->F || tu->shape(2) != L->d || td->shape(0) != L->E ||
        td->shape(1) != L->d || td->shape(2) != L->F) {
        *why = p + "gate/up must be (E, F, d) and down (E, d, F)";
        return false;
    }
    const std::string arch = f.arch();
    int64_t n_exp = L->E;
    f.get_int(arch + ".expert_count", &n_exp);
    if (!f.get_int(arch + ".expert_used_count", &L->n_used)) {
        *why = arch + ".expert_used_count missing; refusing to guess routing";
        return false;
    }
    if (n_exp != L->E) {
        *why = "expert_count disagrees with the expert tensors";
        return false;
    }
    if (L->router && L->router->n_values != L->E * L->d) {
        *why = p + "ffn_gate_inp.weight must be (n_expert, n_embd)";
        return false;
    }
    L->sh_inp = f.find(p + "ffn_gate_inp_shexp.weight");
    L->sh_gate = f.find(p + "ffn_gate_shexp.weight");
    L->sh_up = f.find(p + "ffn_up_shexp.weight");
    L->sh_down = f.find(p + "ffn_down_shexp.weight");
    const aero::GgufTensor *sgi = L->sh_inp, *sg = L->sh_gate, *su = L->sh_up, *sd = L->sh_down;
    if (sg) {
        if (!sgi || !su || !sd || sg->dims.size() != 2 || su->dims.size() != 2 || sd->dims.size() != 2) {
            *why = p + "incomplete shared expert";
            return false;
        }
        L->Fs = sg->shape(0);
        if (sg->shape(1) != L->d || su->shape(0) != L->Fs || su->shape(1) != L->d || sd->shape(0) != L->d ||
            sd->shape(1) != L->Fs || sgi->n_values != L->d) {
            *why = p + "shared expert shapes do not match n_embd";
            return false;
        }
    }
    return true;
}

}  // namespace

extern "C" int aero_cuda_moe_gguf_info(const char* path, int layer, int64_t* out8, char* err, int errlen) {
    aero::GgufFile f;
    std::string why;
    if (!path || !out8) {
        put_err(err, errlen, "null argument");
        return -1;
    }
    LayerTensors L;
    if (!f.open(path, &why) || !find_layer(f, layer, &L, &why)) {
        put_err(err, errlen, why);
        return -1;
    }
    const int64_t v[8] = {L.d, L.E, L.n_used, L.F, L.Fs, L.sh_gate ? 1 : 0, L.gate->type, L.router ? 1 : 0};
    for (int i = 0; i < 8; ++i) out8[i] = v[i];
    return 0;
}

extern "C" void* aero_cuda_moe_open_gguf(const char* path, int layer, int device, int expert_begin, int expert_end,
                                         char* err, int errlen) {
    aero::GgufFile f;
    std::string why;
    if (!path || !f.open(path, &why)) {
        put_err(err, errlen, path ? why : "null path");
        return nullptr;
    }
    LayerTensors L;
    if (!find_layer(f, layer, &L, &why)) {
        put_err(err, errlen, why);
        return nullptr;
    }
    const aero::GgufTensor *tg = L.gate, *tu = L.up, *td = L.down, *tr = L.router;
    const int64_t E = L.E, F = L.F, d = L.d, n_used = L.n_used;
    std::vector<std::pair<void*, size_t>> tmp;
    aero_cuda_moe_desc desc{};
    desc.n_embd = (int)d;
    desc.n_expert = (int)E;
    desc.n_expert_used = (int)n_used;
    desc.ffn_len = (int)F;
    desc.norm_topk_prob = 1;
    desc.device = device;
    desc.expert_begin = expert_begin;
    desc.expert_end = expert_end;
    desc.gate_exps = {tg->type, 0, f.data(*tg), tg->nbytes};
    desc.up_exps = {tu->type, 0, f.data(*tu), tu->nbytes};
    desc.down_exps = {td->type, 0, f.data(*td), td->nbytes};
    void* result = nullptr;
    do {
        if (tr) {
            desc.router = small_f32(f, *tr, device, tmp, &why);
            if (!desc.router) break;
        }
        if (L.sh_gate) {
            desc.has_shared = 1;
            desc.ffn_len_shared = (int)L.Fs;
            desc.shexp_gate_inp = small_f32(f, *L.sh_inp, device, tmp, &why);
            if (!desc.shexp_gate_inp) break;
            desc.shexp_gate = {L.sh_gate->type, 0, f.data(*L.sh_gate), L.sh_gate->nbytes};
            desc.shexp_up = {L.sh_up->type, 0, f.data(*L.sh_up), L.sh_up->nbytes};
            desc.shexp_down = {L.sh_down->type, 0, f.data(*L.sh_down), L.sh_down->nbytes};
        }
        char e2[512] = {0};
        result = aero_cuda_moe_open(&desc, e2, sizeof(e2));
        if (!result) why = e2;
    } while (false);
    for (auto& q : tmp) aero::guarded_free(q.first, q.second, aero::kScratch);
    if (!result) put_err(err, errlen, why);
    return result;
}

// ---------------------------------------------------------------- model table
// Every MoE layer of a GGUF file opened as one table whose forward has the
// reference's aero_moe_fn signature, so a single hook context serves the whole
// block loop (src/model.cpp:166-170, 385-387): aero_model_set_moe(model,
// aero_cuda_moe_model_forward, table).
namespace {
struct MoeModel {
    std::vector<void*> layers;  // null: not a MoE layer
};
}  // namespace

extern "C" void* aero_cuda_moe_model_open_gguf(const char* path, int n_layer, int device, char* err, int errlen) {
    aero::GgufFile f;
    std::string why;
    if (!path || !f.open(path, &why)) {
        put_err(err, errlen, path ? why : "null path");
        return nullptr;
    }
    int64_t nl = n_layer;
    if (nl <= 0 && !f.get_int(f.arch() + ".block_count", &nl)) {
        put_err(err, errlen, f.arch() + ".block_count missing and no layer count given");
        return nullptr;
    }
    if (nl <= 0 || nl > 4096) {
        put_err(err, errlen, "layer count out of range");
        return nullptr;
    }
    auto* m = new MoeModel();
    m->layers.assign((size_t)nl, nullptr);
    int n_moe = 0;
    for (int L = 0; L < (int)nl; ++L) {
        const std::string p = "blk." + std::to_string(L) + ".";
        if (!f.find(p + "ffn_gate_exps.weight") && !f.find(p + "ffn_up_exps.weight") &&
            !f.find(p + "ffn_down_exps.weight"))
            continue;  // a dense (or absent) FFN: the table refuses that layer
        char e2[512] = {0};
        m->layers[(size_t)L] = aero_cuda_moe_open_gguf(path, L, device, 0, 0, e2, sizeof(e2));
        if (!m->layers[(size_t)L]) {
            put_err(err, errlen, "layer " + std::to_string(L) + ": " + e2);
            for (void* h : m->layers)
                if (h) aero_cuda_moe_close(h);
            delete m;
            return nullptr;
        }
        ++n_moe;
    }
    if (n_moe == 0) {
        put_err(err, errlen, "no MoE layer in the file");
        delete m;
        return nullptr;
    }
    return m;
}

extern "C" int aero_cuda_moe_model_forward(void* table, int layer, const float* h, int T, int n_embd, float* out) {
    auto* m = static_cast<MoeModel*>(table);
    if (!m || layer < 0 || layer >= (int)m->layers.size() || !m->layers[(size_t)layer]) return 0;
    return aero_cuda_moe_forward(m->layers[(size_t)layer], layer, h, T, n_embd, out);
}

extern "C" void* aero_cuda_moe_model_layer(void* table, int layer) {
    auto* m = static_cast<MoeModel*>(table);
    if (!m || layer < 0 || layer >= (int)m->layers.size()) return nullptr;
    return m->layers[(size_t)layer];
}

extern "C" void aero_cuda_moe_model_close(void* table) {
    auto* m = static_cast<MoeModel*>(table);
    if (!m) return;
    for (void* h : m->layers)
        if (h) aero_cuda_moe_close(h);
    delete m;
}
