// Engine weight loading by Hugging Face tensor name.
//
// The reference resolves the same names through Candle's VarBuilder
// (src/backends/qwen2.rs:157-159, 234-260, 396-405, 455-465, 592-596).  Here
// q/k/v land in one fused [(Hq + 2 Hkv) * D, H] matrix (one GEMM per layer)
// and gate/up in one [2I, H] matrix; everything is stored in the model dtype.
// Under tensor parallelism the caller passes full tensors and each rank keeps
// its KV-head group of q/k/v rows and o_proj columns, and its slice of the
// gate/up rows and down_proj columns.
#include <cstring>
#include <string>

#include "ms_engine.h"

namespace ms {

namespace {

// Where a named tensor goes: the full source is rows_full x cols elements;
// under tensor parallelism this rank keeps rows [off, off+len) (shard 1) or
// columns [off, off+len) (shard 2) of it.
struct Dest {
  void *ptr = nullptr;
  int64_t rows_full = 0, cols = 0;
  int shard = 0;
  int64_t off = 0, len = 0;
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
  const int64_t r = eng->rank;
  const int64_t hq_f = hq * eng->tp, hkv_f = hkv * eng->tp, I_f = I * eng->tp;
  auto whole = [&](void *ptr, int64_t rows, int64_t cols) { d = Dest{ptr, rows, cols, 0, 0, 0}; };
  auto by_rows = [&](void *ptr, int64_t rows_full, int64_t cols, int64_t len) {
    d = Dest{ptr, rows_full, cols, 1, r * len, len};
  };
  auto by_cols = [&](void *ptr, int64_t rows, int64_t cols_full, int64_t len) {
    d = Dest{ptr, rows, cols_full, 2, r * len, len};
  };
  if (name == "model.embed_tokens.weight") {
    whole(eng->embed, V, H);
  } else if (name == "lm_head.weight") {
    if (eng->cfg.tie_word_embeddings) return eng->fail(MS_E_INVALID, "lm_head.weight given for a tied-embedding config");
    whole(eng->lm_head, V, H);
  } else if (name == "model.norm.weight") {
    whole(eng->final_norm, 1, H);
  } else if (parse_layer(name, layer, suf) && layer >= 0 && layer < eng->L) {
    LayerW &w = eng->layers[layer];
    char *qkv = static_cast<char *>(w.w_qkv);
    char *bqkv = static_cast<char *>(w.b_qkv);
    char *gu = static_cast<char *>(w.w_gu);
    if (suf == "input_layernorm.weight") whole(w.ln1, 1, H);
    else if (suf == "post_attention_layernorm.weight") whole(w.ln2, 1, H);
    else if (suf == "self_attn.q_proj.weight") by_rows(qkv, hq_f * D, H, hq * D);
    else if (suf == "self_attn.k_proj.weight") by_rows(qkv + hq * D * H * es, hkv_f * D, H, hkv * D);
    else if (suf == "self_attn.v_proj.weight") by_rows(qkv + (hq + hkv) * D * H * es, hkv_f * D, H, hkv * D);
    else if (suf == "self_attn.o_proj.weight") by_cols(w.w_o, H, hq_f * D, hq * D);
    else if (suf == "mlp.gate_proj.weight") by_rows(gu, I_f, H, I);
    else if (suf == "mlp.up_proj.weight") by_rows(gu + I * H * es, I_f, H, I);
    else if (suf == "mlp.down_proj.weight") by_cols(w.w_down, H, I_f, I);
    else if (bqkv && suf == "self_attn.q_proj.bias") by_rows(bqkv, hq_f * D, 1, hq * D);
    else if (bqkv && suf == "self_attn.k_proj.bias") by_rows(bqkv + hq * D * es, hkv_f * D, 1, hkv * D);
    else if (bqkv && suf == "self_attn.v_proj.bias") by_rows(bqkv + (hq + hkv) * D * es, hkv_f * D, 1, hkv * D);
    else if (w.q_norm && suf == "self_attn.q_norm.weight") whole(w.q_norm, 1, D);
    else if (w.k_norm && suf == "self_attn.k_norm.weight") whole(w.k_norm, 1, D);
  }
  if (!d.ptr) return eng->fail(MS_E_INVALID, "unknown or unexpected tensor: " + name);
  if (d.rows_full * d.cols != numel)
    return eng->fail(MS_E_INVALID, "tensor " + name + ": expected " + std::to_string(d.rows_full * d.cols) +
                                       " elements, got " + std::to_string(numel));
  cudaError_t e = cudaSetDevice(eng->dev);
  // Order against everything already issued on the device (a device-resident
  // source may come from another stream); the engine stream is non-blocking.
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return eng->fail(MS_E_DEVICE, cudaGetErrorString(e));
  const size_t ses = src_dtype == MS_DTYPE_F32 ? 4 : 2;
  // this rank's part, gathered compactly into a temporary in the source dtype
  const int64_t out_rows = d.shard == 1 ? d.len : d.rows_full;
  const int64_t out_cols = d.shard == 2 ? d.len : d.cols;
  const int64_t n = out_rows * out_cols;
  const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  void *tmp = nullptr;
  e = cudaMalloc(&tmp, size_t(n) * ses);
  if (e == cudaSuccess) {
    const char *src = static_cast<const char *>(data);
    if (d.shard == 2) {
      // stream-ordered: a plain copy from pageable memory may return before its DMA lands
      e = cudaMemcpy2DAsync(tmp, size_t(out_cols) * ses, src + size_t(d.off) * ses, size_t(d.cols) * ses,
                            size_t(out_cols) * ses, size_t(out_rows), kind, eng->stream);
    } else {
      const size_t off = d.shard == 1 ? size_t(d.off) * size_t(d.cols) * ses : 0;
      e = cudaMemcpyAsync(tmp, src + off, size_t(n) * ses, kind, eng->stream);
    }
  }
  if (e == cudaSuccess) {
    if (src_dtype == eng->dtype)
      e = cudaMemcpyAsync(d.ptr, tmp, size_t(n) * ses, cudaMemcpyDeviceToDevice, eng->stream);
    else
      e = launch_convert(tmp, src_dtype, d.ptr, eng->dtype, n, eng->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(eng->stream);
  if (tmp) cudaFree(tmp);
  if (e != cudaSuccess) return eng->fail(MS_E_DEVICE, std::string("weight upload: ") + cudaGetErrorString(e));
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
