// Engine weight loading by Hugging Face tensor name.
//
// The reference resolves the same names through Candle's VarBuilder
// (src/backends/qwen2.rs:157-159, 234-260, 396-405, 455-465, 592-596).  Here
// q/k/v land in one fused [(Hq + 2 Hkv) * D, H] matrix (one GEMM per layer)
// and gate/up in one [2I, H] matrix; everything is stored in the model dtype.
#include <cstring>
#include <string>

#include "ms_engine.h"

namespace ms {

namespace {

struct Dest {
  void *ptr = nullptr;
  int64_t numel = 0;
};

bool parse_layer(const std::string &name, int &layer, std::string &suffix) {
  const std::string pre = "model.layers.";
  if (name.compare(0, pre.size(), pre) != 0) return false;
  size_t i = pre.size(), j = i;
  while (j < name.size() && name[j] >= '0' && name[j] <= '9') ++j;
  if (j == i || j >= name.size() || name[j] != '.') return false;
  layer = std::stoi(name.substr(i, j - i));
  suffix = name.substr(j + 1);
  return true;
}

}  // namespace

int load_weight_impl(Engine *eng, const char *cname, const void *data, int64_t numel, int src_dtype,
                     int src_on_device) {
  if (!cname || !data) return eng->fail(MS_E_INVALID, "null weight name or data");
  if (src_dtype != MS_DTYPE_F32 && src_dtype != MS_DTYPE_BF16 && src_dtype != MS_DTYPE_F16)
    return eng->fail(MS_E_INVALID, "unknown source dtype");
  const std::string name(cname);
  const size_t es = eng->esize;
  const int64_t H = eng->H, I = eng->I, V = eng->V, D = eng->D, hq = eng->hq, hkv = eng->hkv;
  Dest d;
  int layer = -1;
  std::string suf;
  if (name == "model.embed_tokens.weight") {
    d = {eng->embed, V * H};
  } else if (name == "lm_head.weight") {
    if (eng->cfg.tie_word_embeddings) return eng->fail(MS_E_INVALID, "lm_head.weight given for a tied-embedding config");
    d = {eng->lm_head, V * H};
  } else if (name == "model.norm.weight") {
    d = {eng->final_norm, H};
  } else if (parse_layer(name, layer, suf) && layer >= 0 && layer < eng->L) {
    LayerW &w = eng->layers[layer];
    char *qkv = static_cast<char *>(w.w_qkv);
    char *bqkv = static_cast<char *>(w.b_qkv);
    char *gu = static_cast<char *>(w.w_gu);
    if (suf == "input_layernorm.weight") d = {w.ln1, H};
    else if (suf == "post_attention_layernorm.weight") d = {w.ln2, H};
    else if (suf == "self_attn.q_proj.weight") d = {qkv, hq * D * H};
    else if (suf == "self_attn.k_proj.weight") d = {qkv + hq * D * H * es, hkv * D * H};
    else if (suf == "self_attn.v_proj.weight") d = {qkv + (hq + hkv) * D * H * es, hkv * D * H};
    else if (suf == "self_attn.o_proj.weight") d = {w.w_o, H * hq * D};
    else if (suf == "mlp.gate_proj.weight") d = {gu, I * H};
    else if (suf == "mlp.up_proj.weight") d = {gu + I * H * es, I * H};
    else if (suf == "mlp.down_proj.weight") d = {w.w_down, H * I};
    else if (bqkv && suf == "self_attn.q_proj.bias") d = {bqkv, hq * D};
    else if (bqkv && suf == "self_attn.k_proj.bias") d = {bqkv + hq * D * es, hkv * D};
    else if (bqkv && suf == "self_attn.v_proj.bias") d = {bqkv + (hq + hkv) * D * es, hkv * D};
    else if (w.q_norm && suf == "self_attn.q_norm.weight") d = {w.q_norm, D};
    else if (w.k_norm && suf == "self_attn.k_norm.weight") d = {w.k_norm, D};
  }
  if (!d.ptr) return eng->fail(MS_E_INVALID, "unknown or unexpected tensor: " + name);
  if (d.numel != numel)
    return eng->fail(MS_E_INVALID, "tensor " + name + ": expected " + std::to_string(d.numel) + " elements, got " +
                                       std::to_string(numel));
  cudaError_t e = cudaSetDevice(eng->dev);
  // Order against everything already issued on the device (a device-resident
  // source may come from another stream); the engine stream is non-blocking.
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return eng->fail(MS_E_DEVICE, cudaGetErrorString(e));
  const size_t sbytes = size_t(numel) * (src_dtype == MS_DTYPE_F32 ? 4 : 2);
  const void *src = data;
  void *tmp = nullptr;
  if (!src_on_device) {
    // stream-ordered upload: a plain cudaMemcpy from pageable memory may return
    // before its DMA lands, and the copy below runs on the engine stream
    e = cudaMalloc(&tmp, sbytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tmp, data, sbytes, cudaMemcpyHostToDevice, eng->stream);
    if (e != cudaSuccess) {
      if (tmp) cudaFree(tmp);
      return eng->fail(MS_E_DEVICE, std::string("weight upload: ") + cudaGetErrorString(e));
    }
    src = tmp;
  }
  if (src_dtype == eng->dtype)
    e = cudaMemcpyAsync(d.ptr, src, sbytes, cudaMemcpyDeviceToDevice, eng->stream);
  else
    e = launch_convert(src, src_dtype, d.ptr, eng->dtype, numel, eng->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(eng->stream);
  if (tmp) cudaFree(tmp);
  if (e != cudaSuccess) return eng->fail(MS_E_DEVICE, std::string("weight convert: ") + cudaGetErrorString(e));
  eng->loaded[name] += 1;
  return MS_OK;
}

int finalize_impl(Engine *eng) {
  for (const std::string &n : eng->required)
    if (eng->loaded.find(n) == eng->loaded.end()) return eng->fail(MS_E_INVALID, "missing tensor: " + n);
  eng->finalized = true;
  return MS_OK;
}

}  // namespace ms
