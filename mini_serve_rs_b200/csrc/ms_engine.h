// Engine state behind the C ABI of include/ms_engine.h.
#pragma once

#include <cublas_v2.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "ms_internal.h"

namespace ms {

// One admitted request: what CandleBackend keeps per request
// (src/backends/candle.rs:405-418) minus the contiguous KV clone -- its K/V
// now live in the shared paged pool at the scheduler's block ids.
struct Seq {
  int slot = -1;                  // device block-table row
  std::vector<uint32_t> prompt;
  std::vector<int32_t> blocks;    // host mirror of the row
  int synced = 0;                 // leading entries already on the device
  int cached = 0;                 // tokens whose K/V sit in the pool
  bool prefilled = false;
};

struct LayerW {
  void *ln1 = nullptr, *ln2 = nullptr;
  void *w_qkv = nullptr, *b_qkv = nullptr;  // [(Hq+2Hkv)*D, H], [(Hq+2Hkv)*D]
  void *q_norm = nullptr, *k_norm = nullptr;
  void *w_o = nullptr;                      // [H, Hq*D]
  void *w_gu = nullptr;                     // [2I, H]  gate rows then up rows
  void *w_down = nullptr;                   // [H, I]
};

struct Engine {
  ms_model_cfg cfg{};
  ms_engine_opts opts{};
  int dev = 0;
  cudaStream_t stream = nullptr;
  cublasHandle_t blas = nullptr;
  void *blas_ws = nullptr;
  int dtype = MS_DTYPE_BF16;
  size_t esize = 2;
  int D = 128, hq = 0, hkv = 0, H = 0, I = 0, V = 0, L = 0;  // hq, hkv, I: this rank's shard
  int tp = 1, rank = 0;
  void *comm = nullptr;  // ncclComm_t when tp > 1
  int qkv_dim = 0;

  // weights (one allocation)
  void *wbuf = nullptr;
  size_t wbytes = 0;
  void *embed = nullptr, *lm_head = nullptr, *final_norm = nullptr;
  std::vector<LayerW> layers;
  std::unordered_map<std::string, int> loaded;  // name -> times loaded
  std::vector<std::string> required;
  bool finalized = false;

  // RoPE tables [rope_len, D/2] in the model dtype
  void *cos_t = nullptr, *sin_t = nullptr;
  int rope_len = 0;

  // paged pool [L][2][pool_blocks][hkv][16][D]
  void *pool = nullptr;
  size_t pool_bytes = 0;
  size_t layer_pool_elems = 0;  // pool_blocks * hkv * 16 * D

  // tensor-core attention: TMA tensor maps of each layer's K and V pool
  bool use_tc = false;
  std::vector<CUtensorMap> kmaps, vmaps;

  // per-slot device state
  int32_t *d_block_tables = nullptr;  // [max_seqs][max_blocks_per_seq]
  int32_t *d_slot_last = nullptr;     // [max_seqs]
  unsigned *d_status = nullptr;

  // step buffers
  void *sbuf = nullptr;
  size_t sbytes = 0;
  int32_t *d_in = nullptr;  // uploaded step description
  size_t in_cap = 0;        // int32 elements
  int32_t *d_cu = nullptr, *d_pos = nullptr, *d_row_table = nullptr, *d_row_ctx = nullptr;
  int32_t *d_last_index = nullptr, *d_next = nullptr;
  int64_t *d_slots = nullptr;
  void *x_resid = nullptr, *x_norm = nullptr, *x_tmp = nullptr, *qkv = nullptr, *qbuf = nullptr,
       *attn = nullptr, *gu = nullptr, *act = nullptr, *last_norm = nullptr;
  float *logits = nullptr;
  void *attn_ws = nullptr;
  size_t attn_ws_bytes = 0;

  // pinned host staging
  int32_t *h_in = nullptr;
  int32_t *h_next = nullptr;
  unsigned *h_status = nullptr;
  cudaEvent_t done_ev = nullptr;

  // CUDA graphs of pure-decode steps, keyed by (batch, attention partition,
  // context capacity); replayed with a fixed-layout step description
  struct StepGraph {
    int S = 0, part = 0, max_ctx_cap = 0;
    cudaGraphExec_t exec = nullptr;
    int64_t launches = 0;  // kernels per replay
    uint64_t last_use = 0;
  };
  bool graphs_enabled = true;
  std::vector<StepGraph> graphs;
  std::unordered_map<int64_t, int> graph_warm;  // (S, part) -> eager steps run
  uint64_t graph_clock = 0;
  int64_t graph_captures = 0, graph_replays = 0;
  int32_t *d_gin = nullptr, *h_gin = nullptr;  // fixed graph staging, graph_in_elems(max_seqs)
  void drop_graphs() {
    for (auto &g : graphs)
      if (g.exec) cudaGraphExecDestroy(g.exec);
    graphs.clear();
    graph_warm.clear();
  }

  // tensor parallelism: peer-mapped partial-sum buffers for the fused
  // all-reduce + residual add + RMSNorm (ms_tp_allreduce.cu)
  bool ar_fused = false;
  bool ar_capable = false;              // the peer mappings exist (fused setup agreed by all ranks)
  void *ar_sym = nullptr;               // own allocation: 2 partial-sum buffers + signal array
  void *ar_buf[2][8] = {};              // [buffer][rank]
  uint32_t *ar_sig[8] = {};             // each rank's signal array
  std::vector<void *> ar_peer_maps;     // IPC mappings to close
  uint32_t ar_epoch = 0;

  // instrumentation
  int64_t kernel_launches = 0;
  int64_t last_launches = 0;  // kernels enqueued by the last enqueue_forward
  bool profiling = false;
  std::vector<cudaEvent_t> prof_ev;  // pairs: start, end
  size_t prof_used = 0;              // events in use (2 per bracketed launch)
  double prof_bytes = 0.0;
  // debugging: >= 0 ends the layer loop after that layer's MLP down
  // projection (no lm_head, no sampling), so the activation buffers hold it
  int debug_stop_layer = -1;
  // tensor parallelism: pairs around each all-reduce + residual add + RMSNorm
  // (the fused kernel, or NCCL all-reduce + K4)
  std::vector<cudaEvent_t> prof_ar_ev;
  size_t prof_ar_used = 0;

  // host bookkeeping
  std::unordered_map<uint64_t, Seq> seqs;
  std::vector<int> free_slots;
  bool healthy = true;
  int inject = 0;
  std::string err;

  // last step
  bool pending = false;
  int last_nseq = 0, last_T = 0, last_max_ctx = 0;
  std::vector<int> last_slots;
  std::vector<uint8_t> last_flags;
  std::vector<uint64_t> last_ids;
  int last_in = 0;             // sequences listed in the last step description
  std::vector<int> last_map;   // listed index -> packed row, -1 when not run
  std::vector<uint8_t> last_out_flags;  // per listed sequence

  int fail(int code, const std::string &msg) {
    err = msg;
    if (code == MS_E_DEVICE || code == MS_E_INJECTED) quarantine();
    return code;
  }
  void quarantine() {
    // candle.rs:689-696: a BackendError clears every request's state
    healthy = false;
    seqs.clear();
    free_slots.clear();
    for (int i = opts.max_seqs - 1; i >= 0; --i) free_slots.push_back(i);
    pending = false;
  }
};

// implemented across ms_engine*.cu
// create_impl fills a caller-allocated Engine; destroy_impl releases its
// device resources (the caller deletes the object).
int create_impl(const ms_model_cfg *cfg, const ms_engine_opts *opts, Engine *eng);
void destroy_impl(Engine *eng);
int load_weight_impl(Engine *eng, const char *name, const void *data, int64_t numel, int src_dtype,
                     int src_on_device);
int finalize_impl(Engine *eng);
int seq_admit_impl(Engine *eng, uint64_t id, const uint32_t *prompt, int prompt_len, const int32_t *blocks,
                   int nblocks, int num_cached);
int seq_append_block_impl(Engine *eng, uint64_t id, int32_t block);
int seq_release_impl(Engine *eng, uint64_t id);
int step_launch_impl(Engine *eng, const ms_step_desc *desc);

// What one step's device work needs to know (host-computed, uploaded rows).
struct StepPlan {
  int S = 0, T = 0, nd = 0;  // sequences, packed tokens, block-table deltas
  int n_dec = 0;             // rows run by the decode kernel (row list uploaded when tiles are used)
  int n_tiles = 0;           // prefill tiles (tensor-core path only)
  bool nucleus = false;      // some sampled row has 0 < top_p < 1 (always set for a graph step)
  int max_ctx_dec = 0;
  long long blocks_dec = 0;  // sum over decode rows of pages read
  double ctx_dec = 0.0;      // sum over decode rows of keys read
  bool split = false;        // decode rows via row list + prefill tiles
  // decode attention launch shape
  int part = 1;              // pages per split-K partition
  int max_ctx_launch = 0;    // grid sized for contexts up to this (>= max_ctx_dec)
  // step description: pinned host staging -> device, one copy
  //   [hdr][row S][ntok S][start S][tok T]([temp S][top_p S][seed_lo S][seed_hi S] when sample)
  //   [drow dc][didx dc][dblk dc][dec n_dec][tiles 4 n_tiles]
  const int32_t *h_desc = nullptr;
  int32_t *d_desc = nullptr;
  size_t desc_elems = 0;
  int hdr = 0;               // leading words; with graph, word 0 = the delta count
  int delta_cap = 0;         // dc: capacity of the delta arrays
  bool graph = false;        // fixed layout read by a replayed graph
  bool sample = false;       // per-row sampling parameters staged, sampling kernel launched
};
// Elements of the fixed graph staging for batches up to max_seqs.
inline size_t graph_in_elems(int max_seqs) { return 4 + size_t(11) * max_seqs; }
// Split-K partition size of the decode attention for a step (the same for the
// eager and the graph path, so both produce identical results).
int decode_partition(const Engine *eng, const StepPlan &plan, int max_ctx);
int enqueue_forward(Engine *eng, const StepPlan &plan);
int tp_fused_setup(Engine *eng);
void tp_fused_teardown(Engine *eng);
cudaError_t launch_ar_add_rmsnorm(Engine *eng, int which, const void *residual, const int32_t *row_index,
                                  const void *w, void *resid_out, void *norm_out, int rows, cudaStream_t st);
int step_wait_impl(Engine *eng, uint32_t *out_tokens, uint8_t *out_flags);

}  // namespace ms
