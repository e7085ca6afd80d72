// Deferred weight gradients and packed-operand attachments.
//
// Semantics of the reference's DeferredHostJob / AsyncDwPolicy
// (torch_xdna_device.cpp:299-482, 550-656, 1212-1250): convolution_backward
// returns the weight gradient before computing it; the storage carries the
// pending job; the first reader (the optimizer, a copy, any op) runs it; a
// gradient freed unread drops its job without ever running it.  The job owns
// snapshots of its operands (the packed X and dY rows), so later in-place
// changes of x or dy do not leak into dW.
//
// On B200 "running" a job means enqueueing its wgrad kernel on the current
// stream, so a reader never blocks the host; stream order makes every later
// kernel see the finished gradient.  With XDNA_ASYNC_DW=1 (default) the
// policy learns K = dX calls per optimizer step and, once two steps agree,
// launches all pending jobs right after the K-th dX of a step instead of
// waiting for a reader.
#include <algorithm>
#include <cstdlib>
#include <unordered_map>
#include <vector>

#include "xdna.h"

namespace xdna {

std::atomic<int64_t> g_pending_jobs{0};

namespace {

struct Job {
  std::function<void()> fn;
  int64_t order = 0;
  bool kick = true;  // launched early by the async policy (weight gradients)
};

struct Attachment {
  at::Tensor rows;
  int64_t version = 0;
  std::vector<int64_t> sizes, strides;
  int64_t offset = 0;
};

// A packed (GEMM-operand) form of a weight, valid while the weight's version,
// geometry and storage are unchanged and nothing wrote the storage.
struct WeightSlot {
  int kind = 0;
  int64_t version = 0;
  std::vector<int64_t> sizes, strides;
  int64_t offset = 0;
  at::Tensor packed;
};

std::mutex g_mu;
std::unordered_map<void*, Job> g_jobs;               // storage data ptr -> pending job
std::unordered_map<void*, Attachment> g_attach;      // storage data ptr -> packed rows
std::unordered_map<void*, std::vector<WeightSlot>> g_wslots;  // storage data ptr -> packed weights
std::atomic<int64_t> g_nwslots{0};
int64_t g_whits = 0, g_wmisses = 0;

// pending outputs with foldable tails, and the storages their producers read
struct EpiSlot {
  std::shared_ptr<EpiSpec> spec;
  std::vector<int64_t> sizes, strides;
  int64_t offset = 0;
  std::vector<void*> inputs;
};
std::unordered_map<void*, EpiSlot> g_epi;            // output storage -> slot
// gated BatchNorm outputs (storage -> source and the output's geometry)
struct GateSlot {
  std::shared_ptr<GateSource> src;
  std::vector<int64_t> sizes, strides;
  int64_t offset = 0;
};
std::unordered_map<void*, GateSlot> g_gates;
std::atomic<int64_t> g_ngates{0};
std::unordered_multimap<void*, void*> g_readers;     // input storage -> pending output storage
std::atomic<int64_t> g_nreaders{0};
int64_t g_folded = 0;

// Moves the slot of `out` out of the tables (destroyed by the caller, outside
// the lock: it may hold the last reference to a tensor).
EpiSlot take_epi_locked(void* out) {
  EpiSlot slot;
  auto it = g_epi.find(out);
  if (it == g_epi.end()) return slot;
  slot = std::move(it->second);
  g_epi.erase(it);
  for (void* in : slot.inputs) {
    auto range = g_readers.equal_range(in);
    for (auto r = range.first; r != range.second;) {
      if (r->second == out) r = g_readers.erase(r);
      else ++r;
    }
  }
  g_nreaders.store(int64_t(g_readers.size()));
  return slot;
}
int64_t g_order = 0;
int64_t g_started = 0, g_dropped = 0, g_kicks = 0, g_deferred = 0;
int64_t g_dx_this_step = 0, g_k_prev = -1, g_k_learned = 0;

bool async_enabled() {
  static const bool on = [] {
    const char* s = std::getenv("XDNA_ASYNC_DW");
    return !s || std::string(s) != "0";
  }();
  return on;
}

void run_job(std::function<void()>& fn) {
  fn();
}

}  // namespace

// Entries are always moved out of the tables before they are destroyed:
// destroying a job or an attachment frees tensors, and the allocator's release
// hook (on_release) takes g_mu again.
void defer_write(const at::Tensor& target, std::function<void()> job, bool kick) {
  void* key = target.storage().mutable_data();
  Job old;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_jobs.find(key);
    if (it != g_jobs.end()) old = std::move(it->second);
    g_jobs[key] = Job{std::move(job), g_order++, kick};
    ++g_deferred;
    g_pending_jobs.store(int64_t(g_jobs.size()));
  }
}

namespace {
void materialize_key(void* key) {
  std::function<void()> fn;
  EpiSlot slot;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_jobs.find(key);
    if (it == g_jobs.end()) return;
    fn = std::move(it->second.fn);
    g_jobs.erase(it);
    ++g_started;
    g_pending_jobs.store(int64_t(g_jobs.size()));
    slot = take_epi_locked(key);
  }
  run_job(fn);
}
}  // namespace

void drop_pending(const at::Tensor& t) {
  if (g_pending_jobs.load(std::memory_order_relaxed) == 0 || !t.defined() || !t.has_storage()) return;
  void* key = t.storage().mutable_data();
  Job done;
  EpiSlot slot;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_jobs.find(key);
    if (it == g_jobs.end()) return;
    done = std::move(it->second);
    g_jobs.erase(it);
    ++g_started;
    g_pending_jobs.store(int64_t(g_jobs.size()));
    slot = take_epi_locked(key);
  }
}

void materialize(const at::Tensor& t) {
  if (g_pending_jobs.load(std::memory_order_relaxed) == 0 || !t.defined() || !t.has_storage()) return;
  materialize_key(t.storage().mutable_data());
}

void defer_epilogue(const at::Tensor& out, const std::vector<at::Tensor>& inputs, std::shared_ptr<EpiSpec> spec,
                    std::function<void()> job) {
  // a producer with a spec waits for its reader (that is its point); only the
  // weight-gradient jobs (no spec) go with the async policy's early launch
  const bool kick = spec == nullptr;
  defer_write(out, std::move(job), kick);
  void* key = out.storage().mutable_data();
  std::lock_guard<std::mutex> lk(g_mu);
  EpiSlot& slot = g_epi[key];
  slot.spec = std::move(spec);
  slot.sizes = out.sizes().vec();
  slot.strides = out.strides().vec();
  slot.offset = out.storage_offset();
  for (const at::Tensor& in : inputs) {
    if (!in.defined() || !in.has_storage()) continue;
    void* ik = in.storage().mutable_data();
    slot.inputs.push_back(ik);
    g_readers.emplace(ik, key);
  }
  g_nreaders.store(int64_t(g_readers.size()));
}

std::shared_ptr<EpiSpec> find_epilogue(const at::Tensor& t) {
  if (g_pending_jobs.load(std::memory_order_relaxed) == 0 || !t.defined() || !t.has_storage()) return nullptr;
  void* key = t.storage().mutable_data();
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_epi.find(key);
  if (it == g_epi.end() || !g_jobs.count(key)) return nullptr;
  const EpiSlot& s = it->second;
  if (s.sizes != t.sizes().vec() || s.strides != t.strides().vec() || s.offset != t.storage_offset()) return nullptr;
  return s.spec;
}

void note_folded() {
  std::lock_guard<std::mutex> lk(g_mu);
  ++g_folded;
}

void add_epilogue_input(const at::Tensor& out, const at::Tensor& input) {
  if (!input.defined() || !input.has_storage()) return;
  void* key = out.storage().mutable_data();
  void* ik = input.storage().mutable_data();
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_epi.find(key);
  if (it == g_epi.end()) return;
  it->second.inputs.push_back(ik);
  g_readers.emplace(ik, key);
  g_nreaders.store(int64_t(g_readers.size()));
}

void before_write(const at::Tensor& t) {
  if (g_nreaders.load(std::memory_order_relaxed) == 0 || !t.defined() || !t.has_storage()) return;
  std::vector<void*> outs;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto range = g_readers.equal_range(t.storage().mutable_data());
    for (auto r = range.first; r != range.second; ++r) outs.push_back(r->second);
  }
  for (void* o : outs) materialize_key(o);
}

bool has_pending(const at::Tensor& t) {
  if (g_pending_jobs.load() == 0 || !t.defined() || !t.has_storage()) return false;
  std::lock_guard<std::mutex> lk(g_mu);
  return g_jobs.count(t.storage().mutable_data()) != 0;
}

void materialize_all() {
  std::vector<std::pair<int64_t, std::function<void()>>> fns;
  std::unordered_map<void*, EpiSlot> slots;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto& kv : g_jobs) fns.emplace_back(kv.second.order, std::move(kv.second.fn));
    g_started += int64_t(g_jobs.size());
    g_jobs.clear();
    g_pending_jobs.store(0);
    slots.swap(g_epi);
    g_readers.clear();
    g_nreaders.store(0);
  }
  std::sort(fns.begin(), fns.end(), [](auto& a, auto& b) { return a.first < b.first; });
  for (auto& f : fns) run_job(f.second);
}

void on_release(void* ptr) {
  if (!ptr) return;
  Job dropped;
  Attachment att;
  std::vector<WeightSlot> slots;
  EpiSlot epi;
  GateSlot gate;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto gs = g_gates.find(ptr);
    if (gs != g_gates.end()) {
      gate = std::move(gs->second);
      g_gates.erase(gs);
      g_ngates.store(int64_t(g_gates.size()));
    }
    auto ws = g_wslots.find(ptr);
    if (ws != g_wslots.end()) {
      slots = std::move(ws->second);
      g_wslots.erase(ws);
      g_nwslots.store(int64_t(g_wslots.size()));
    }
    epi = take_epi_locked(ptr);
    auto it = g_jobs.find(ptr);
    if (it != g_jobs.end()) {
      dropped = std::move(it->second);
      g_jobs.erase(it);
      ++g_dropped;
      g_pending_jobs.store(int64_t(g_jobs.size()));
    }
    auto at = g_attach.find(ptr);
    if (at != g_attach.end()) {
      att = std::move(at->second);
      g_attach.erase(at);
    }
  }
}

void note_gate_source(void* storage_data, std::vector<int64_t> sizes, std::vector<int64_t> strides, int64_t offset,
                      std::shared_ptr<GateSource> src) {
  if (!storage_data) return;
  GateSlot fresh{std::move(src), std::move(sizes), std::move(strides), offset};
  GateSlot old;
  std::lock_guard<std::mutex> lk(g_mu);
  GateSlot& slot = g_gates[storage_data];
  old = std::move(slot);
  slot = std::move(fresh);
  g_ngates.store(int64_t(g_gates.size()));
}

std::shared_ptr<GateSource> find_gate_source(const at::Tensor& y) {
  if (g_ngates.load(std::memory_order_relaxed) == 0 || !y.defined() || !y.has_storage()) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_gates.find(y.storage().mutable_data());
  if (it == g_gates.end()) return nullptr;
  const GateSlot& s = it->second;
  if (s.sizes != y.sizes().vec() || s.strides != y.strides().vec() || s.offset != y.storage_offset()) return nullptr;
  return s.src;
}

void note_dgrad() {
  bool kick = false;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    ++g_dx_this_step;
    kick = async_enabled() && g_k_learned > 0 && g_dx_this_step == g_k_learned && !g_jobs.empty();
    if (kick) ++g_kicks;
  }
  if (!kick) return;
  // the pending weight gradients, in the order they were deferred
  std::vector<std::pair<int64_t, std::function<void()>>> fns;
  std::vector<EpiSlot> slots;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto it = g_jobs.begin(); it != g_jobs.end();) {
      if (!it->second.kick) {
        ++it;
        continue;
      }
      fns.emplace_back(it->second.order, std::move(it->second.fn));
      slots.push_back(take_epi_locked(it->first));
      ++g_started;
      it = g_jobs.erase(it);
    }
    g_pending_jobs.store(int64_t(g_jobs.size()));
  }
  std::sort(fns.begin(), fns.end(), [](auto& a, auto& b) { return a.first < b.first; });
  for (auto& f : fns) run_job(f.second);
}

void note_optimizer_step() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_dx_this_step > 0) {
    if (g_dx_this_step == g_k_prev) g_k_learned = g_dx_this_step;
    g_k_prev = g_dx_this_step;
  }
  g_dx_this_step = 0;
}

std::map<std::string, int64_t> deferred_stats() {
  std::lock_guard<std::mutex> lk(g_mu);
  return {{"pending", int64_t(g_jobs.size())}, {"deferred", g_deferred}, {"started", g_started},
          {"dropped", g_dropped},          {"kicks", g_kicks},       {"k_learned", g_k_learned},
          {"attached_rows", int64_t(g_attach.size())}, {"packed_weights", int64_t(g_wslots.size())},
          {"packed_weight_hits", g_whits}, {"packed_weight_misses", g_wmisses},
          {"folded_tails", g_folded}, {"pending_tails", int64_t(g_epi.size())},
          {"gated_outputs", int64_t(g_gates.size())}};
}

void note_write(const at::Tensor& t) {
  if (g_nwslots.load(std::memory_order_relaxed) == 0 || !t.defined() || !t.has_storage()) return;
  std::vector<WeightSlot> dropped;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_wslots.find(t.storage().mutable_data());
  if (it == g_wslots.end()) return;
  dropped = std::move(it->second);
  g_wslots.erase(it);
  g_nwslots.store(int64_t(g_wslots.size()));
}

at::Tensor find_packed_weight(const at::Tensor& w, int kind) {
  if (!w.has_storage()) return {};
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_wslots.find(w.storage().mutable_data());
  if (it != g_wslots.end())
    for (const WeightSlot& ws : it->second)
      if (ws.kind == kind && ws.version == int64_t(w._version()) && ws.sizes == w.sizes().vec() &&
          ws.strides == w.strides().vec() && ws.offset == w.storage_offset()) {
        ++g_whits;
        return ws.packed;
      }
  ++g_wmisses;
  return {};
}

void attach_packed_weight(const at::Tensor& w, int kind, const at::Tensor& packed) {
  if (!w.has_storage()) return;
  WeightSlot fresh{kind, int64_t(w._version()), w.sizes().vec(), w.strides().vec(), w.storage_offset(), packed};
  WeightSlot old;
  std::lock_guard<std::mutex> lk(g_mu);
  auto& v = g_wslots[w.storage().mutable_data()];
  for (WeightSlot& ws : v)
    if (ws.kind == kind) {
      old = std::move(ws);
      ws = std::move(fresh);
      return;
    }
  v.push_back(std::move(fresh));
  g_nwslots.store(int64_t(g_wslots.size()));
}

void attach_rows(const at::Tensor& input, const at::Tensor& rows) {
  if (!input.has_storage()) return;
  Attachment old;
  Attachment fresh{rows, int64_t(input._version()), input.sizes().vec(), input.strides().vec(),
                   input.storage_offset()};
  std::lock_guard<std::mutex> lk(g_mu);
  auto& slot = g_attach[input.storage().mutable_data()];
  old = std::move(slot);
  slot = std::move(fresh);
}

at::Tensor find_rows(const at::Tensor& input) {
  if (!input.has_storage()) return {};
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_attach.find(input.storage().mutable_data());
  if (it == g_attach.end()) return {};
  const Attachment& a = it->second;
  if (a.version != int64_t(input._version()) || a.sizes != input.sizes().vec() ||
      a.strides != input.strides().vec() || a.offset != input.storage_offset())
    return {};
  return a.rows;
}

}  // namespace xdna
