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

}  // namespace

extern "C" void* aero_cuda_moe_open_gguf(const char* path, int layer, int device, int expert_begin, int expert_end,
                                         char* err, int errlen) {
    aero::GgufFile f;
    std::string why;
    if (!path || !f.open(path, &why)) {
        put_err(err, errlen, path ? why : "null path");
        return nullptr;
    }
    const std::string p = "blk." + std::to_string(layer) + ".";
    const aero::GgufTensor* tg = f.find(p + "ffn_gate_exps.weight");
    const aero::GgufTensor* tu = f.find(p + "ffn_up_exps.weight");
    const aero::GgufTensor* td = f.find(p + "ffn_down_exps.weight");
    const aero::GgufTensor* tr = f.find(p + "ffn_gate_inp.weight");
    if (!tg || !tu || !td) {
        put_err(err, errlen, p + "ffn_{gate,up,down}_exps.weight missing: not a MoE layer");
        return nullptr;
    }
    if (tg->dims.size() != 3 || tu->dims.size() != 3 || td->dims.size() != 3) {
        put_err(err, errlen, p + "expert tensors must be 3-D (n_expert, out, in)");
        return nullptr;
    }
    const int64_t E = tg->shape(0), F = tg->shape(1), d = tg->shape(2);
    if (tu->shape(0) != E || tu->shape(1) != F || tu->shape(2) != d || td->shape(0) != E || td->shape(1) != d ||
        td->shape(2) != F) {
        put_err(err, errlen, p + "gate/up must be (E, F, d) and down (E, d, F)");
        return nullptr;
    }
    const std::string arch = f.arch();
    int64_t n_exp = E, n_used = -1;
    f.get_int(arch + ".expert_count", &n_exp);
    if (!f.get_int(arch + ".expert_used_count", &n_used)) {
        put_err(err, errlen, arch + ".expert_used_count missing; refusing to guess routing");
        return nullptr;
    }
    if (n_exp != E) {
        put_err(err, errlen, "expert_count disagrees with the expert tensors");
        return nullptr;
    }
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
            if (tr->n_values != E * d) {
                why = p + "ffn_gate_inp.weight must be (n_expert, n_embd)";
                break;
            }
            desc.router = small_f32(f, *tr, device, tmp, &why);
            if (!desc.router) break;
        }
        const aero::GgufTensor* sgi = f.find(p + "ffn_gate_inp_shexp.weight");
        const aero::GgufTensor* sg = f.find(p + "ffn_gate_shexp.weight");
        const aero::GgufTensor* su = f.find(p + "ffn_up_shexp.weight");
        const aero::GgufTensor* sd = f.find(p + "ffn_down_shexp.weight");
        if (sg) {
            if (!sgi || !su || !sd || sg->dims.size() != 2 || su->dims.size() != 2 || sd->dims.size() != 2) {
                why = p + "incomplete shared expert";
                break;
            }
            const int64_t Fs = sg->shape(0);
            if (sg->shape(1) != d || su->shape(0) != Fs || su->shape(1) != d || sd->shape(0) != d || sd->shape(1) != Fs ||
                sgi->n_values != d) {
                why = p + "shared expert shapes do not match n_embd";
                break;
            }
            desc.has_shared = 1;
            desc.ffn_len_shared = (int)Fs;
            desc.shexp_gate_inp = small_f32(f, *sgi, device, tmp, &why);
            if (!desc.shexp_gate_inp) break;
            desc.shexp_gate = {sg->type, 0, f.data(*sg), sg->nbytes};
            desc.shexp_up = {su->type, 0, f.data(*su), su->nbytes};
            desc.shexp_down = {sd->type, 0, f.data(*sd), sd->nbytes};
        }
        char e2[512] = {0};
        result = aero_cuda_moe_open(&desc, e2, sizeof(e2));
        if (!result) why = e2;
    } while (false);
    for (auto& q : tmp) aero::guarded_free(q.first, q.second, aero::kScratch);
    if (!result) put_err(err, errlen, why);
    return result;
}
