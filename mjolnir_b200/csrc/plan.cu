// Host-side split-KV planner and the runner handle of the C ABI.
//
// mj_plan_split_kv is the planner of mjolnir_b200/plan.py in C++, for hosts
// that drive the library without Python: the reference's occupancy-pinned
// split (arch/thor/plan.py:140-197: one wave holds sm_count * ctas_per_sm /
// (h_k * n_q_tiles) work items; a batch smaller than a wave gets the smallest
// chunk whose items fit one wave; items longest first, padded with empty items
// for a fixed grid) plus the B200 rebalance (the cheapest of that chunk and
// every ceil(T / k), k = 1 .. max_splits, under a longest-first model of the
// persistent grid's rounds plus a per-item overhead). Both produce the same
// plans for the same inputs (checked against each other in the tests).
//
// mj_runner owns what a decode step needs besides the caller's tensors: the
// fixed-address work list and split counts (so a captured CUDA graph replays
// later plans), the split-KV partials, the device status word, and a pinned
// staging copy of the plan. It allocates only in mj_create.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <set>
#include <vector>

#include "common.cuh"

namespace mj {
int set_last_error(int code, const char* msg);
}

namespace {

struct Item {
  int32_t seq, tb, te, split;
};

int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// Longest-first wave model of the decode time, in tile units.
double wave_cost(const std::vector<int>& tiles, int chunk, int slots, double item_overhead) {
  std::vector<int> lens;
  int kmax = 0;
  for (int t : tiles) {
    const int k = ceil_div(t, chunk);
    kmax = std::max(kmax, k);
    for (int j = 0; j + 1 < k; ++j) lens.push_back(chunk);
    lens.push_back(t - (k - 1) * chunk);
  }
  std::sort(lens.begin(), lens.end(), [](int a, int b) { return a > b; });
  double sum = 0.0;
  int waves = 0;
  for (size_t i = 0; i < lens.size(); i += (size_t)slots) {
    sum += lens[i];
    ++waves;
  }
  return sum + item_overhead * waves + (kmax > 1 ? 0.25 : 0.0);
}

}  // namespace

struct mj_runner {
  int device, h_q, h_k, head_size, page_size, max_num_seqs, max_q_len, kv_format, max_splits, ctas_per_sm, sm_count;
  int cap;  // work-list capacity (fixed-grid length)
  int32_t* work = nullptr;      // device (cap, 4)
  int32_t* n_splits = nullptr;  // device (max_num_seqs,)
  float* o_part = nullptr;      // device partials
  float* lse_part = nullptr;
  int32_t* status = nullptr;    // device status word
  int32_t* stage = nullptr;     // pinned host staging: work then n_splits
  cudaEvent_t staged = nullptr; // the last plan's copy out of the staging buffer
  // the last plan
  int num_seqs = 0, q_len = 0, num_work = 0, with_reduction = 0, chunk_tiles = 0;
};

extern "C" {

int mj_plan_split_kv(const int32_t* seq_lens, int num_seqs, int h_k, int n_q_tiles, int sm_count, int ctas_per_sm,
                     int max_splits, int pad_to, int rebalance, float item_overhead, int32_t* work_out,
                     int work_capacity, int32_t* n_splits_out, int* num_work_out, int* chunk_tiles_out) {
  if (!seq_lens || num_seqs <= 0 || h_k <= 0 || n_q_tiles <= 0 || sm_count <= 0 || ctas_per_sm <= 0 || max_splits <= 0 ||
      !work_out || !n_splits_out || !num_work_out)
    return mj::set_last_error(MJ_ERR_INVALID, "mj_plan_split_kv: invalid argument");
  std::vector<int> tiles(num_seqs);
  int T = 1;
  for (int b = 0; b < num_seqs; ++b) {
    tiles[b] = std::max(1, ceil_div(std::max(seq_lens[b], 0), mj::kTileRows));
    T = std::max(T, tiles[b]);
  }
  const int slots = std::max(1, (sm_count * ctas_per_sm) / (h_k * n_q_tiles));
  const int shortest = std::max(1, ceil_div(T, max_splits));  // cap chunks per sequence
  int chunk = T;
  if (max_splits > 1) {
    // the reference's chunk: none when the batch fills a round, else the
    // shortest chunk whose items fit in one round
    if (num_seqs < slots) {
      int lo = shortest, hi = T;
      while (lo < hi) {
        const int mid = (lo + hi) / 2;
        int64_t items = 0;
        for (int t : tiles) items += ceil_div(t, mid);
        if (items <= slots) hi = mid;
        else lo = mid + 1;
      }
      chunk = lo;
    }
    if (rebalance) {  // the cheapest of it and every ceil(T / k) under the round model
      std::set<int> cset{chunk};
      for (int k = 1; k <= max_splits; ++k) cset.insert(std::max(shortest, ceil_div(T, k)));
      double best = 0.0;
      bool have = false;
      for (auto it = cset.rbegin(); it != cset.rend(); ++it) {  // longest chunk first: it keeps a tie
        const double cost = wave_cost(tiles, *it, slots, item_overhead);
        if (!have || cost < best - 1e-9) {
          best = cost;
          chunk = *it;
          have = true;
        }
      }
    }
  }
  std::vector<Item> work;
  for (int b = 0; b < num_seqs; ++b) {
    const int k = ceil_div(tiles[b], chunk);
    n_splits_out[b] = k;
    for (int j = 0; j < k; ++j) work.push_back({b, j * chunk, std::min((j + 1) * chunk, tiles[b]), j});
  }
  std::stable_sort(work.begin(), work.end(), [](const Item& x, const Item& y) { return (x.te - x.tb) > (y.te - y.tb); });
  const int n = (int)work.size();
  const int total = pad_to > 0 ? pad_to : n;
  if (pad_to > 0 && pad_to < n) return mj::set_last_error(MJ_ERR_INVALID, "mj_plan_split_kv: pad_to below the work items");
  if (total > work_capacity) return mj::set_last_error(MJ_ERR_INVALID, "mj_plan_split_kv: work_out too small");
  for (int i = 0; i < total; ++i) {
    const Item w = i < n ? work[i] : Item{0, 0, 0, 0};
    work_out[4 * i + 0] = w.seq;
    work_out[4 * i + 1] = w.tb;
    work_out[4 * i + 2] = w.te;
    work_out[4 * i + 3] = w.split;
  }
  *num_work_out = total;
  if (chunk_tiles_out) *chunk_tiles_out = chunk;
  return MJ_OK;
}

// ---- runner handle --------------------------------------------------------

// the tensor-core kernel's rows per job (48; 16 at head_size 256) and CTAs
// per SM (the configured count up to 16 rows at head_size 128; else one)
static int runner_n_tiles(const mj_runner* r, int q_len) {
  const int n_q = q_len * (r->h_q / r->h_k);
  const int rows = r->head_size == 256 ? 16 : 48;
  return n_q <= rows ? 1 : (n_q + rows - 1) / rows;
}
static int runner_ctas(const mj_runner* r, int q_len) {
  return q_len * (r->h_q / r->h_k) <= 16 && r->head_size == 128 ? r->ctas_per_sm : 1;
}

void mj_destroy(mj_runner* r) {
  if (!r) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(r->device);
  if (r->staged) {
    cudaEventSynchronize(r->staged);
    cudaEventDestroy(r->staged);
  }
  cudaFree(r->work);
  cudaFree(r->n_splits);
  cudaFree(r->o_part);
  cudaFree(r->lse_part);
  cudaFree(r->status);
  cudaFreeHost(r->stage);
  cudaSetDevice(prev);
  delete r;
}

mj_runner* mj_create(int device, int h_q, int h_k, int head_size, int page_size, int max_num_seqs, int max_q_len,
                     int kv_format, int max_splits, int ctas_per_sm) {
  if (h_q <= 0 || h_k <= 0 || h_q % h_k || head_size <= 0 || page_size <= 0 || max_num_seqs <= 0 || max_q_len <= 0 ||
      max_splits <= 0 || ctas_per_sm <= 0 || mj_row_bytes(head_size, kv_format) < 0) {
    mj::set_last_error(MJ_ERR_INVALID, "mj_create: invalid shape or format");
    return nullptr;
  }
  if (max_q_len * (h_q / h_k) > 64) {
    mj::set_last_error(MJ_ERR_UNSUPPORTED, "mj_create: more than 64 query rows per KV head");
    return nullptr;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  mj_runner* r = new mj_runner();
  r->device = device;
  r->h_q = h_q;
  r->h_k = h_k;
  r->head_size = head_size;
  r->page_size = page_size;
  r->max_num_seqs = max_num_seqs;
  r->max_q_len = max_q_len;
  r->kv_format = kv_format;
  r->max_splits = max_splits;
  r->ctas_per_sm = ctas_per_sm;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&r->sm_count, cudaDevAttrMultiProcessorCount, device);
  const int slots1 = std::max(1, (r->sm_count * runner_ctas(r, 1)) / (h_k * runner_n_tiles(r, 1)));
  r->cap = std::max(max_num_seqs * max_splits, slots1);
  const int64_t nq = (int64_t)max_q_len * (h_q / h_k);
  const int64_t rows = (int64_t)max_splits * max_num_seqs * h_k * nq;
  if (e == cudaSuccess) e = cudaMalloc(&r->work, (size_t)r->cap * 4 * sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMalloc(&r->n_splits, (size_t)max_num_seqs * sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMalloc(&r->o_part, (size_t)rows * head_size * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&r->lse_part, (size_t)rows * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&r->status, sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMemset(r->status, 0, sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMemset(r->work, 0, (size_t)r->cap * 4 * sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMallocHost(&r->stage, ((size_t)r->cap * 4 + max_num_seqs) * sizeof(int32_t));
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->staged, cudaEventDisableTiming);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "mj_create: %s", cudaGetErrorString(e));
    mj::set_last_error(MJ_ERR_CUDA, msg);
    mj_destroy(r);
    return nullptr;
  }
  return r;
}

int mj_plan(mj_runner* r, const int32_t* seq_lens_host, int num_seqs, int q_len, int margin, int fixed_grid,
            void* stream) {
  if (!r || !seq_lens_host) return mj::set_last_error(MJ_ERR_INVALID, "mj_plan: null argument");
  if (num_seqs <= 0 || num_seqs > r->max_num_seqs || q_len < 1 || q_len > r->max_q_len || margin < 0)
    return mj::set_last_error(MJ_ERR_INVALID, "mj_plan: num_seqs / q_len beyond the runner's capacity");
  // the previous plan's copy must have left the staging buffer
  cudaError_t e = cudaEventSynchronize(r->staged);
  if (e != cudaSuccess) return mj::set_last_error(MJ_ERR_CUDA, cudaGetErrorString(e));
  std::vector<int32_t> lens(seq_lens_host, seq_lens_host + num_seqs);
  for (auto& L : lens) L += margin;
  int32_t* work_h = r->stage;
  int32_t* ns_h = r->stage + (size_t)r->cap * 4;
  int num_work = 0, chunk = 0;
  int rc = mj_plan_split_kv(lens.data(), num_seqs, r->h_k, runner_n_tiles(r, q_len), r->sm_count, runner_ctas(r, q_len),
                            r->max_splits, r->cap, 1, 2.0f, work_h, r->cap, ns_h, &num_work, &chunk);
  if (rc) return rc;
  int real = 0, most = 1;
  for (int i = 0; i < num_work; ++i) real += work_h[4 * i + 2] > work_h[4 * i + 1];
  for (int b = 0; b < num_seqs; ++b) most = std::max(most, (int)ns_h[b]);
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(r->device);
  cudaStream_t s = (cudaStream_t)stream;
  e = cudaMemcpyAsync(r->work, work_h, (size_t)r->cap * 4 * sizeof(int32_t), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(r->n_splits, ns_h, (size_t)num_seqs * sizeof(int32_t), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaEventRecord(r->staged, s);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return mj::set_last_error(MJ_ERR_CUDA, cudaGetErrorString(e));
  r->num_seqs = num_seqs;
  r->q_len = q_len;
  r->num_work = fixed_grid ? r->cap : real;
  r->with_reduction = (most > 1 || fixed_grid) ? 1 : 0;
  r->chunk_tiles = chunk;
  return MJ_OK;
}

int mj_runner_fill(const mj_runner* r, mj_decode_args* a) {
  if (!r || !a) return mj::set_last_error(MJ_ERR_INVALID, "mj_runner_fill: null argument");
  if (!r->num_seqs) return mj::set_last_error(MJ_ERR_INVALID, "mj_runner_fill: no plan yet (call mj_plan)");
  a->num_seqs = r->num_seqs;
  a->q_len = r->q_len;
  a->h_q = r->h_q;
  a->h_k = r->h_k;
  a->head_size = r->head_size;
  a->page_size = r->page_size;
  a->kv_format = r->kv_format;
  a->work = r->work;
  a->num_work = r->num_work;
  a->n_splits = r->n_splits;
  a->max_splits = r->max_splits;
  a->o_part = r->o_part;
  a->lse_part = r->lse_part;
  a->part_seqs = r->max_num_seqs;
  a->with_combine = r->with_reduction;
  a->status = r->status;
  return MJ_OK;
}

int mj_runner_status(mj_runner* r) {
  if (!r) return -mj::set_last_error(MJ_ERR_INVALID, "mj_runner_status: null runner");
  int32_t code = 0;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(r->device);
  cudaError_t e = cudaMemcpy(&code, r->status, sizeof(int32_t), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && code) e = cudaMemset(r->status, 0, sizeof(int32_t));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return -mj::set_last_error(MJ_ERR_CUDA, cudaGetErrorString(e));
  return code;
}

}  // extern "C"
