// Native serving runtime: paged-KV block manager with prefix caching and a
// continuous-batching scheduler with chunked prefill.
//
// Reference behaviour: rlx-serve src/batch.rs:370-560 (`ContinuousBatcher::
// {admit, pump, advance_seq}` over rlx_runtime::paged_kv::BatchConstructor:
// token budget + max entries, prefill/decode queues, chunked prefill) and
// rlx-models-core src/prompt_cache.rs:54-240 (longest-prefix KV reuse). Here
// the KV lives in fixed 16-token device blocks; the scheduler emits, per step,
// the flat token batch (ids, positions, cache slots) plus block tables and
// context lengths straight into pinned host staging buffers, so the Python
// side does one host->device copy per field and launches the model.
//
// Policy per step:
//   1. every running sequence that has finished its prompt gets one decode
//      token (allocating a new block at a block boundary; if the pool is
//      empty the most recently admitted sequence is preempted and will be
//      recomputed),
//   2. the remaining token budget goes to prefill chunks: first sequences
//      whose prompt is partially computed, then new admissions (FIFO) while
//      the sequence limit and free blocks allow.
// Overlapped (asynchronous) scheduling: when schedule() is given a `tok_src`
// buffer, every sampled row appends a placeholder token to its sequence at
// once, so step n+1 can be scheduled and launched while step n still runs on
// the GPU. A decode row whose input is such a placeholder gets tok_src[t] =
// the logit row of the previous step that produces it (the device copies the
// token from the previous step's sampler output); update() later replaces
// placeholders, oldest first, by the sampled values. A sequence whose
// placeholders already reach max_new_tokens is not scheduled again; one that
// stops on EOS / a stop id discards the row that was scheduled behind it.
// Prefix caching: every full block is keyed by a chained 64-bit hash of its
// tokens; freed blocks that carry a hash stay reusable (LRU) until the pool
// needs them, and an admitted prompt skips its longest cached block prefix.
#include <torch/extension.h>

#include <algorithm>
#include <cstdint>
#include <deque>
#include <list>
#include <memory>
#include <optional>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace b200rt {

constexpr int kBlock = 16;

static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static uint64_t block_hash(uint64_t prev, const int32_t* toks) {
  uint64_t h = mix64(prev ^ 0x5bd1e995ull);
  for (int i = 0; i < kBlock; ++i) h = mix64(h ^ (uint64_t)(uint32_t)toks[i] ^ ((uint64_t)i << 40));
  return h;
}

class BlockManager {
 public:
  BlockManager(int num_blocks, bool prefix_caching)
      : num_blocks_(num_blocks), prefix_caching_(prefix_caching), ref_(num_blocks, 0), hash_(num_blocks, 0),
        has_hash_(num_blocks, 0) {
    for (int b = num_blocks - 1; b >= 0; --b) free_.push_back(b);
  }
  int num_free() const { return (int)free_.size() + (int)lru_.size(); }
  int num_blocks() const { return num_blocks_; }

  int allocate() {
    int b;
    if (!free_.empty()) {
      b = free_.back();
      free_.pop_back();
    } else if (!lru_.empty()) {
      b = lru_.front();
      lru_.pop_front();
      lru_pos_.erase(b);
      if (has_hash_[b]) {
        auto it = cached_.find(hash_[b]);
        if (it != cached_.end() && it->second == b) cached_.erase(it);
        has_hash_[b] = 0;
      }
    } else {
      return -1;
    }
    ref_[b] = 1;
    return b;
  }

  void release(int b) {
    if (--ref_[b] > 0) return;
    if (prefix_caching_ && has_hash_[b]) {
      lru_.push_back(b);
      lru_pos_[b] = std::prev(lru_.end());
    } else {
      has_hash_[b] = 0;
      free_.push_back(b);
    }
  }

  // Register a full block's hash (first writer wins).
  void publish(int b, uint64_t h) {
    if (!prefix_caching_) return;
    if (cached_.count(h)) return;
    cached_[h] = b;
    hash_[b] = h;
    has_hash_[b] = 1;
  }

  // Look up a cached block; on hit take a reference.
  int acquire_cached(uint64_t h) {
    if (!prefix_caching_) return -1;
    auto it = cached_.find(h);
    if (it == cached_.end()) return -1;
    const int b = it->second;
    if (ref_[b] == 0) {
      auto p = lru_pos_.find(b);
      if (p != lru_pos_.end()) {
        lru_.erase(p->second);
        lru_pos_.erase(p);
      }
    }
    ++ref_[b];
    return b;
  }

  // Cached block of a hash without taking a reference (-1 if absent).
  int peek_cached(uint64_t h) const {
    if (!prefix_caching_) return -1;
    auto it = cached_.find(h);
    return it == cached_.end() ? -1 : it->second;
  }

  int64_t hits = 0, queries = 0;

 private:
  int num_blocks_;
  bool prefix_caching_;
  std::vector<int> ref_;
  std::vector<uint64_t> hash_;
  std::vector<uint8_t> has_hash_;
  std::vector<int> free_;
  std::list<int> lru_;
  std::unordered_map<int, std::list<int>::iterator> lru_pos_;
  std::unordered_map<uint64_t, int> cached_;
};

enum Status { WAITING = 0, RUNNING = 1, FINISHED = 2 };

struct Seq {
  int64_t id;
  std::vector<int32_t> tokens;
  int prompt_len;
  int num_computed = 0;
  int max_new_tokens;
  bool ignore_eos;
  std::vector<int32_t> stop_ids;
  std::vector<int32_t> blocks;
  std::vector<uint64_t> hashes;  // chained hash of each full, published block
  int status = WAITING;
  int finish_reason = 0;  // 1 length, 2 stop token, 3 aborted
  int num_cached_prompt = 0;
  int pending = 0;        // trailing placeholder tokens whose values the device has not returned yet
  int pending_row = -1;   // logit row (of the step that made it) of the newest placeholder
  bool length_done = false;  // placeholders reach max_new_tokens: finishes when they resolve
  int generated() const { return (int)tokens.size() - prompt_len; }
  int resolved_generated() const { return (int)tokens.size() - pending - prompt_len; }
};

class Scheduler {
 public:
  Scheduler(int num_blocks, int max_num_seqs, int max_batched_tokens, int max_blocks_per_seq, bool prefix_caching,
            int chunk_size)
      : bm_(num_blocks, prefix_caching),
        max_num_seqs_(max_num_seqs),
        budget_(max_batched_tokens),
        max_blocks_per_seq_(max_blocks_per_seq),
        chunk_(chunk_size > 0 ? chunk_size : max_batched_tokens) {}

  int64_t add_request(const std::vector<int32_t>& prompt, int max_new_tokens, bool ignore_eos,
                      const std::vector<int32_t>& stop_ids) {
    if (prompt.empty()) throw std::invalid_argument("empty prompt");
    const int need = ((int)prompt.size() + max_new_tokens + kBlock - 1) / kBlock;
    if (need > max_blocks_per_seq_) throw std::invalid_argument("request longer than the model context");
    auto s = std::make_unique<Seq>();
    s->id = next_id_++;
    s->tokens = prompt;
    s->prompt_len = (int)prompt.size();
    s->max_new_tokens = max_new_tokens;
    s->ignore_eos = ignore_eos;
    s->stop_ids = stop_ids;
    waiting_.push_back(s->id);
    seqs_[s->id] = std::move(s);
    return next_id_ - 1;
  }

  void abort(int64_t id) {
    auto it = seqs_.find(id);
    if (it == seqs_.end() || it->second->status == FINISHED) return;
    finish(*it->second, 3);
  }

  bool has_work() const { return !waiting_.empty() || !running_.empty(); }
  int num_waiting() const { return (int)waiting_.size(); }
  int num_running() const { return (int)running_.size(); }
  int num_free_blocks() const { return bm_.num_free(); }

  // Build the next step into the pinned staging buffers. Returns a dict with
  // counts; the per-row sequence ids to sample are written to `sample_ids`.
  py::dict schedule(torch::Tensor input_ids, torch::Tensor positions, torch::Tensor slots,
                    torch::Tensor dec_tables, torch::Tensor dec_ctx, torch::Tensor pre_tables, torch::Tensor pre_ctx,
                    torch::Tensor pre_cu, torch::Tensor logit_rows, torch::Tensor sample_ids,
                    std::optional<torch::Tensor> tok_src_opt, bool overlap) {
    const bool has_src = tok_src_opt.has_value() && tok_src_opt->numel() > 0;
    if (overlap && !has_src) throw std::invalid_argument("scheduler: overlapped scheduling needs tok_src");
    int32_t* tsrc = has_src ? tok_src_opt->data_ptr<int32_t>() : nullptr;
    if (has_src && tok_src_opt->numel() < input_ids.numel())
      throw std::invalid_argument("scheduler: tok_src must hold as many rows as input_ids");
    int32_t* ids = input_ids.data_ptr<int32_t>();
    int32_t* pos = positions.data_ptr<int32_t>();
    int64_t* slt = slots.data_ptr<int64_t>();
    int32_t* dtab = dec_tables.data_ptr<int32_t>();
    int32_t* dctx = dec_ctx.data_ptr<int32_t>();
    int32_t* ptab = pre_tables.data_ptr<int32_t>();
    int32_t* pctx = pre_ctx.data_ptr<int32_t>();
    int32_t* pcu = pre_cu.data_ptr<int32_t>();
    int64_t* lrows = logit_rows.data_ptr<int64_t>();
    int64_t* sids = sample_ids.data_ptr<int64_t>();
    const int64_t cap_tok = input_ids.numel();
    const int64_t cap_seq = dec_ctx.numel();
    const int W = (int)dec_tables.size(1);

    step_decode_.clear();
    step_prefill_.clear();
    int tokens = 0;

    // 1. decode tokens for running sequences past their prompt
    std::vector<int64_t> decoders;
    for (int64_t id : running_) {
      const Seq& s = *seqs_[id];
      if (is_decode(s) && !s.length_done) decoders.push_back(id);
    }
    for (size_t i = 0; i < decoders.size(); ++i) {
      Seq& s = *seqs_[decoders[i]];
      if (s.status != RUNNING) continue;
      while (!ensure_slots(s, s.num_computed + 1)) {
        if (!preempt_last(s.id)) break;
      }
      if (s.status != RUNNING) continue;
      if ((int)s.blocks.size() * kBlock < s.num_computed + 1) continue;  // could not allocate
      if (tokens >= budget_ || tokens >= cap_tok || (int64_t)step_decode_.size() >= cap_seq) break;
      step_decode_.push_back(s.id);
      ++tokens;
    }
    // a sequence preempted while the loop above allocated for a later one drops out
    step_decode_.erase(std::remove_if(step_decode_.begin(), step_decode_.end(),
                                      [&](int64_t id) { return seqs_[id]->status != RUNNING; }),
                       step_decode_.end());
    tokens = (int)step_decode_.size();
    // longest context first: the decode attention grid walks rows in order, so the
    // longest (sequence, kv-head) CTAs start in the first wave and short ones fill the tail
    std::stable_sort(step_decode_.begin(), step_decode_.end(),
                     [&](int64_t x, int64_t y) { return seqs_[x]->num_computed > seqs_[y]->num_computed; });
    // 2. prefill chunks (continuing sequences first, then admissions)
    std::vector<int64_t> cand;
    for (int64_t id : running_) {
      Seq& s = *seqs_[id];
      if (s.status == RUNNING && !is_decode(s) && s.pending == 0 && s.num_computed < prefill_limit(s))
        cand.push_back(id);
    }
    std::vector<int> chunk_len;
    for (int64_t id : cand) {
      if (tokens >= budget_) break;
      Seq& s = *seqs_[id];
      int n = std::min({prefill_limit(s) - s.num_computed, budget_ - tokens, chunk_});
      if (!ensure_slots(s, s.num_computed + n)) {
        n = (int)s.blocks.size() * kBlock - s.num_computed;
        if (n <= 0) continue;
      }
      step_prefill_.push_back(id);
      chunk_len.push_back(n);
      tokens += n;
    }
    while (!waiting_.empty() && tokens < budget_ && (int)running_.size() < max_num_seqs_ &&
           (int64_t)(step_decode_.size() + step_prefill_.size()) < cap_seq) {
      Seq& s = *seqs_[waiting_.front()];
      if (s.pending > 0) break;  // preempted with a token still in flight: re-admit once it resolves
      // prefix cache lookup over full prompt blocks (leave >= 1 token to compute)
      if (s.blocks.empty()) {
        uint64_t h = 0;
        const int full = ((int)s.tokens.size() - 1) / kBlock;
        for (int b = 0; b < full; ++b) {
          const uint64_t hb = block_hash(h, s.tokens.data() + b * kBlock);
          ++bm_.queries;
          const int blk = bm_.acquire_cached(hb);
          if (blk < 0) break;
          ++bm_.hits;
          s.blocks.push_back(blk);
          s.hashes.push_back(hb);
          h = hb;
        }
        s.num_computed = (int)s.blocks.size() * kBlock;
        s.num_cached_prompt = s.num_computed;
      }
      const int remaining = prefill_limit(s) - s.num_computed;
      const int n = std::min({remaining, budget_ - tokens, chunk_});
      // keep one block of headroom per running sequence for decode growth
      const int need_blocks = (s.num_computed + n + kBlock - 1) / kBlock - (int)s.blocks.size();
      if (need_blocks > bm_.num_free()) {
        if (s.num_computed > 0 && s.status == WAITING && step_prefill_.empty() && step_decode_.empty() &&
            running_.empty()) {
          // nothing else can free memory: fall through with what we have
        }
        break;
      }
      if (!ensure_slots(s, s.num_computed + n)) break;
      waiting_.pop_front();
      s.status = RUNNING;
      running_.push_back(s.id);
      step_prefill_.push_back(s.id);
      chunk_len.push_back(n);
      tokens += n;
    }
    if (tokens > cap_tok) throw std::runtime_error("scheduler: token staging buffer too small");

    // 3. write the flat batch: decode tokens first, then prefill chunks
    int t = 0, r = 0;
    for (size_t i = 0; i < step_decode_.size(); ++i) {
      Seq& s = *seqs_[step_decode_[i]];
      const int p = s.num_computed;
      const bool placeholder = p >= (int)s.tokens.size() - s.pending;
      ids[t] = placeholder ? 0 : s.tokens[p];
      if (tsrc) tsrc[t] = placeholder ? s.pending_row : -1;
      pos[t] = p;
      slt[t] = (int64_t)s.blocks[p / kBlock] * kBlock + p % kBlock;
      for (int b = 0; b < W; ++b) dtab[i * W + b] = b < (int)s.blocks.size() ? s.blocks[b] : 0;
      dctx[i] = p + 1;
      lrows[r] = t;
      sids[r] = s.id;
      ++r;
      ++t;
    }
    int max_q = 0;
    pcu[0] = 0;
    for (size_t i = 0; i < step_prefill_.size(); ++i) {
      Seq& s = *seqs_[step_prefill_[i]];
      const int n = chunk_len[i];
      for (int j = 0; j < n; ++j) {
        const int p = s.num_computed + j;
        ids[t] = s.tokens[p];
        if (tsrc) tsrc[t] = -1;
        pos[t] = p;
        slt[t] = (int64_t)s.blocks[p / kBlock] * kBlock + p % kBlock;
        ++t;
      }
      for (int b = 0; b < W; ++b) ptab[i * W + b] = b < (int)s.blocks.size() ? s.blocks[b] : 0;
      pctx[i] = s.num_computed + n;
      pcu[i + 1] = pcu[i] + n;
      max_q = std::max(max_q, n);
      if (s.num_computed + n == (int)s.tokens.size()) {  // prompt complete: sample the first token
        lrows[r] = t - 1;
        sids[r] = s.id;
        ++r;
      }
    }
    // advance computed counters (KV for these tokens is written by this step)
    for (int64_t id : step_decode_) seqs_[id]->num_computed += 1;
    for (size_t i = 0; i < step_prefill_.size(); ++i) {
      Seq& s = *seqs_[step_prefill_[i]];
      s.num_computed += chunk_len[i];
      publish_full_blocks(s);
    }
    if (overlap) {
      // every sampled row appends a placeholder now, so the next step can be scheduled before this one returns
      for (int i = 0; i < r; ++i) {
        Seq& s = *seqs_[sids[i]];
        s.tokens.push_back(0);
        ++s.pending;
        s.pending_row = i;
        if (s.generated() >= s.max_new_tokens) s.length_done = true;
      }
    }
    py::dict d;
    d["num_tokens"] = t;
    d["num_decode"] = (int)step_decode_.size();
    d["num_prefill"] = (int)step_prefill_.size();
    d["max_q_len"] = max_q;
    d["num_logits"] = r;
    return d;
  }

  // Ids of every sequence in the last schedule() batch, in batch order
  // (decode rows first, then prefill chunks): per-sequence state slots key on these.
  std::vector<int64_t> step_seq_ids() const {
    std::vector<int64_t> ids(step_decode_);
    ids.insert(ids.end(), step_prefill_.begin(), step_prefill_.end());
    return ids;
  }

  // Append sampled tokens (one per logit row, in schedule() order). Returns
  // the ids of sequences that finished in this update.
  std::vector<int64_t> update(const std::vector<int64_t>& seq_ids, const std::vector<int32_t>& toks, int32_t eos) {
    std::vector<int64_t> done;
    for (size_t i = 0; i < seq_ids.size(); ++i) {
      auto it = seqs_.find(seq_ids[i]);
      if (it == seqs_.end()) continue;
      Seq& s = *it->second;
      if (s.status == FINISHED) continue;  // (a sequence preempted with a token in flight still resolves it)
      if (s.pending > 0) {  // resolve the oldest placeholder
        s.tokens[s.tokens.size() - s.pending] = toks[i];
        --s.pending;
      } else {
        s.tokens.push_back(toks[i]);
      }
      int reason = 0;
      if (s.resolved_generated() >= s.max_new_tokens) reason = 1;
      if (!s.ignore_eos) {
        if (eos >= 0 && toks[i] == eos) reason = 2;
        for (int32_t st : s.stop_ids)
          if (toks[i] == st) reason = 2;
      }
      if (reason) {
        s.tokens.resize(s.tokens.size() - s.pending);  // rows scheduled behind a stop are discarded
        s.pending = 0;
        finish(s, reason);
        done.push_back(s.id);
      }
    }
    return done;
  }

  // Prompt-cache persistence. prefix_blocks: the cached blocks holding the
  // longest full-block prefix of `tokens` (block ids in order; stops at the first
  // block that is not cached). import_prefix: allocate blocks for the full-block
  // prefix of `tokens`, register their hashes and leave them free-but-cached
  // (LRU), so a later request with that prefix reuses them; returns the block ids
  // whose contents the caller must fill (blocks already cached are skipped and
  // returned as -1).
  std::vector<int32_t> prefix_blocks(const std::vector<int32_t>& tokens) const {
    std::vector<int32_t> out;
    uint64_t h = 0;
    const int full = (int)tokens.size() / kBlock;
    for (int b = 0; b < full; ++b) {
      h = block_hash(h, tokens.data() + b * kBlock);
      const int blk = bm_.peek_cached(h);
      if (blk < 0) break;
      out.push_back(blk);
    }
    return out;
  }

  std::vector<int32_t> import_prefix(const std::vector<int32_t>& tokens) {
    std::vector<int32_t> out;
    uint64_t h = 0;
    const int full = (int)tokens.size() / kBlock;
    for (int b = 0; b < full; ++b) {
      h = block_hash(h, tokens.data() + b * kBlock);
      if (bm_.peek_cached(h) >= 0) {
        out.push_back(-1);
        continue;
      }
      const int blk = bm_.allocate();
      if (blk < 0) break;
      bm_.publish(blk, h);
      bm_.release(blk);  // ref 0 with a hash: reusable cached block (LRU)
      out.push_back(blk);
    }
    return out;
  }

  std::vector<int32_t> output_tokens(int64_t id) const {
    const Seq& s = *seqs_.at(id);
    return std::vector<int32_t>(s.tokens.begin() + s.prompt_len, s.tokens.end());
  }
  int finish_reason(int64_t id) const { return seqs_.at(id)->finish_reason; }
  int num_cached_prompt_tokens(int64_t id) const { return seqs_.at(id)->num_cached_prompt; }
  void release(int64_t id) { seqs_.erase(id); }
  py::dict stats() const {
    py::dict d;
    d["prefix_hits"] = bm_.hits;
    d["prefix_queries"] = bm_.queries;
    d["free_blocks"] = bm_.num_free();
    d["num_blocks"] = bm_.num_blocks();
    d["preemptions"] = preemptions_;
    return d;
  }

 private:
  // A running sequence decodes when exactly one known token is not yet cached
  // and it has generated at least one token. Otherwise it prefills up to
  // prefill_limit: the whole prompt for a fresh sequence (its last position
  // yields the first sampled token), or all but the last known token for a
  // sequence re-admitted after preemption (the last one is then decoded).
  static bool is_decode(const Seq& s) {
    return (int)s.tokens.size() > s.prompt_len && (int)s.tokens.size() - s.num_computed == 1;
  }
  static int prefill_limit(const Seq& s) {
    return (int)s.tokens.size() > s.prompt_len ? (int)s.tokens.size() - 1 : (int)s.tokens.size();
  }

  bool ensure_slots(Seq& s, int n_tokens) {
    const int need = (n_tokens + kBlock - 1) / kBlock;
    while ((int)s.blocks.size() < need) {
      const int b = bm_.allocate();
      if (b < 0) return false;
      s.blocks.push_back(b);
    }
    return true;
  }

  void publish_full_blocks(Seq& s) {
    const int full = std::min(s.num_computed, (int)s.tokens.size()) / kBlock;
    while ((int)s.hashes.size() < full) {
      const int b = (int)s.hashes.size();
      const uint64_t prev = b ? s.hashes[b - 1] : 0;
      const uint64_t h = block_hash(prev, s.tokens.data() + b * kBlock);
      s.hashes.push_back(h);
      bm_.publish(s.blocks[b], h);
    }
  }

  void free_blocks(Seq& s) {
    for (int b : s.blocks) bm_.release(b);
    s.blocks.clear();
    s.hashes.clear();
  }

  void finish(Seq& s, int reason) {
    if (s.status == WAITING) waiting_.erase(std::remove(waiting_.begin(), waiting_.end(), s.id), waiting_.end());
    running_.erase(std::remove(running_.begin(), running_.end(), s.id), running_.end());
    s.status = FINISHED;
    s.finish_reason = reason;
    free_blocks(s);
  }

  // Preempt the most recently admitted running sequence other than `keep`
  // (recompute policy: its KV is dropped and it re-enters the waiting queue).
  bool preempt_last(int64_t keep) {
    for (auto it = running_.rbegin(); it != running_.rend(); ++it) {
      if (*it == keep) continue;
      Seq& v = *seqs_[*it];
      free_blocks(v);
      v.num_computed = 0;
      v.status = WAITING;
      waiting_.push_front(v.id);
      running_.erase(std::next(it).base());
      ++preemptions_;
      return true;
    }
    return false;
  }

  BlockManager bm_;
  int max_num_seqs_, budget_, max_blocks_per_seq_, chunk_;
  int64_t next_id_ = 0;
  int64_t preemptions_ = 0;
  std::unordered_map<int64_t, std::unique_ptr<Seq>> seqs_;
  std::deque<int64_t> waiting_;
  std::vector<int64_t> running_;
  std::vector<int64_t> step_decode_, step_prefill_;
};

}  // namespace b200rt

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace b200rt;
  m.doc() = "rlx_models_b200 native serving runtime (block manager + scheduler)";
  py::class_<Scheduler>(m, "Scheduler")
      .def(py::init<int, int, int, int, bool, int>(), py::arg("num_blocks"), py::arg("max_num_seqs"),
           py::arg("max_batched_tokens"), py::arg("max_blocks_per_seq"), py::arg("prefix_caching") = true,
           py::arg("chunk_size") = 0)
      .def("add_request", &Scheduler::add_request, py::arg("prompt"), py::arg("max_new_tokens"),
           py::arg("ignore_eos") = false, py::arg("stop_ids") = std::vector<int32_t>{})
      .def("abort", &Scheduler::abort)
      .def("has_work", &Scheduler::has_work)
      .def("num_waiting", &Scheduler::num_waiting)
      .def("num_running", &Scheduler::num_running)
      .def("num_free_blocks", &Scheduler::num_free_blocks)
      .def("schedule", &Scheduler::schedule, py::arg("input_ids"), py::arg("positions"), py::arg("slots"),
           py::arg("dec_tables"), py::arg("dec_ctx"), py::arg("pre_tables"), py::arg("pre_ctx"), py::arg("pre_cu"),
           py::arg("logit_rows"), py::arg("sample_ids"), py::arg("tok_src") = py::none(),
           py::arg("overlap") = false)
      .def("step_seq_ids", &Scheduler::step_seq_ids)
      .def("update", &Scheduler::update)
      .def("output_tokens", &Scheduler::output_tokens)
      .def("prefix_blocks", &Scheduler::prefix_blocks)
      .def("import_prefix", &Scheduler::import_prefix)
      .def("finish_reason", &Scheduler::finish_reason)
      .def("num_cached_prompt_tokens", &Scheduler::num_cached_prompt_tokens)
      .def("release", &Scheduler::release)
      .def("stats", &Scheduler::stats);
}
