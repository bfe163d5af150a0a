// Native host runtime of mesh_b200 (module mesh_b200._runtime, pybind11).
//
// * PageAllocator   - KV page pool free list (lowest ids first, double-free detection).
// * DecodeScheduler - the fair decode queue and microbatch builder of the serving engine: tasks
//   ordered by (decode_steps_served, fairness_epoch, session id); a batch starts from an optional
//   primary session, then admits queued sessions that share the primary's execution class, stay
//   in the same fast-path token ceiling, keep the KV-length skew inside the runtime mode's
//   guardrail, and fit the batch-size and total-KV budgets; everything else is deferred with a
//   reason count. Semantics follow the reference coordinator
//   (agent/src/inference/coordinator.rs:731-760 enqueue, :992-1250 build_next_decode_batch,
//   :1467-1496 allows_batch_sequence_skew).
// * Serving frame header codec - the 49-byte big-endian tensor-plane header of the reference
//   (agent/src/network/tensor_message.rs:71-218), for the TCP plane used by CPU ranks and
//   cross-host transfers.
// * Ring chunk plan - send/recv chunk indices of a ring reduce-scatter / all-gather step
//   (agent/src/executor/ring_allreduce.rs:1444-1488).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <map>
#include <queue>
#include <set>
#include <stdexcept>
#include <string>
#include <tuple>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace py = pybind11;

namespace mesh_rt {

// ------------------------------------------------------------------------------------------------
class PageAllocator {
 public:
  PageAllocator(int64_t num_pages, int64_t reserved) : num_pages_(num_pages), reserved_(reserved) {
    if (num_pages <= reserved || reserved < 0) throw std::invalid_argument("page pool too small");
    for (int64_t p = reserved; p < num_pages; ++p) free_.push(p);
  }
  py::object alloc(int64_t n) {
    if (n < 0) throw std::invalid_argument("negative page count");
    if ((int64_t)free_.size() < n) return py::none();
    std::vector<int64_t> out;
    out.reserve(n);
    for (int64_t i = 0; i < n; ++i) {
      int64_t p = free_.top();
      free_.pop();
      used_.insert(p);
      out.push_back(p);
    }
    return py::cast(out);
  }
  void free(const std::vector<int64_t>& pages) {
    for (int64_t p : pages) {
      auto it = used_.find(p);
      if (it == used_.end()) throw std::invalid_argument("double free or foreign page " + std::to_string(p));
      used_.erase(it);
      free_.push(p);
    }
  }
  int64_t num_free() const { return (int64_t)free_.size(); }
  int64_t num_used() const { return (int64_t)used_.size(); }
  int64_t capacity() const { return num_pages_ - reserved_; }

 private:
  int64_t num_pages_, reserved_;
  std::priority_queue<int64_t, std::vector<int64_t>, std::greater<int64_t>> free_;
  std::unordered_set<int64_t> used_;
};

// ------------------------------------------------------------------------------------------------
enum RuntimeMode : int { FIT_FIRST = 0, THROUGHPUT_FIRST = 1, LATENCY_FIRST = 2, RESILIENT_EDGE = 3 };

inline bool allows_skew(int mode, int64_t min_kv, int64_t max_kv) {
  if (min_kv == 0 || max_kv <= min_kv) return true;
  switch (mode) {
    case THROUGHPUT_FIRST: return max_kv <= std::max(min_kv * 2, min_kv + 512);
    case LATENCY_FIRST: return max_kv <= std::max((min_kv * 3 + 1) / 2, min_kv + 256);
    default: return true;
  }
}

inline bool requires_bucket_cohesion(int mode) { return mode == THROUGHPUT_FIRST || mode == LATENCY_FIRST; }

struct SessionInfo {
  int64_t class_key = 0;       // provider/profile/executor contract identity
  int64_t kv_tokens = 0;       // logical KV tokens the next decode step attends
  int64_t token_ceiling = -1;  // fast-path decode bucket ceiling (-1: no fast path)
  int mode = THROUGHPUT_FIRST;
  int64_t decode_steps_served = 0;
  bool queued = false;
  bool complete = false;
};

struct Task {
  int64_t steps, epoch, sid;
  bool operator<(const Task& o) const { return std::tie(steps, epoch, sid) < std::tie(o.steps, o.epoch, o.sid); }
};

class DecodeScheduler {
 public:
  void register_session(int64_t sid, int64_t class_key, int64_t kv_tokens, int64_t token_ceiling, int mode) {
    SessionInfo& s = sessions_[sid];
    s.class_key = class_key;
    s.kv_tokens = kv_tokens;
    s.token_ceiling = token_ceiling;
    s.mode = mode;
  }
  void update(int64_t sid, int64_t kv_tokens, int64_t token_ceiling) {
    SessionInfo& s = get(sid);
    s.kv_tokens = kv_tokens;
    s.token_ceiling = token_ceiling;
  }
  void set_complete(int64_t sid, bool c) { get(sid).complete = c; }
  void served(int64_t sid) { ++get(sid).decode_steps_served; }
  int64_t steps_served(int64_t sid) { return get(sid).decode_steps_served; }

  // Queue a session for its next decode step; a session is queued at most once.
  bool enqueue(int64_t sid) {
    SessionInfo& s = get(sid);
    if (s.queued || s.complete) return false;
    ++next_epoch_;
    s.queued = true;
    Task t{s.decode_steps_served, next_epoch_, sid};
    queue_.insert(t);
    index_[sid] = t;
    return true;
  }
  void remove(int64_t sid) {
    auto it = index_.find(sid);
    if (it != index_.end()) {
      queue_.erase(it->second);
      index_.erase(it);
    }
    auto s = sessions_.find(sid);
    if (s != sessions_.end()) s->second.queued = false;
  }
  void drop(int64_t sid) {
    remove(sid);
    sessions_.erase(sid);
  }
  std::vector<int64_t> queued() const {
    std::vector<int64_t> out;
    for (auto& t : queue_) out.push_back(t.sid);
    return out;
  }
  size_t queue_len() const { return queue_.size(); }

  // Build the next microbatch. Returns dict(slots=[(sid, epoch, kv)], deferred=[(sid, epoch)],
  // total_kv_tokens, deferred_for_capacity, deferred_for_kv_budget, deferred_for_guardrail).
  // Deferred sessions stay queued (with their fairness position); admitted ones are dequeued.
  py::dict build_batch(int64_t primary, int64_t max_batch, int64_t max_total_kv) {
    if (max_batch < 1) max_batch = 1;
    if (max_total_kv < 1) max_total_kv = 1;
    std::vector<std::tuple<int64_t, int64_t, int64_t>> slots;
    std::vector<std::pair<int64_t, int64_t>> deferred;
    int64_t total = 0, d_cap = 0, d_kv = 0, d_guard = 0;
    int64_t bmin = -1, bmax = -1;
    bool have_class = false;
    int64_t cls = 0, ceiling = -1;
    int mode = THROUGHPUT_FIRST;
    std::vector<Task> ordered(queue_.begin(), queue_.end());
    std::vector<int64_t> admitted;

    auto it_primary = index_.find(primary);
    if (primary >= 0 && it_primary != index_.end()) {
      Task t = it_primary->second;
      SessionInfo& s = get(t.sid);
      if (!s.complete) {
        have_class = true;
        cls = s.class_key;
        mode = s.mode;
        ceiling = s.token_ceiling;
        slots.emplace_back(t.sid, t.epoch, s.kv_tokens);
        bmin = bmax = s.kv_tokens;
        total += s.kv_tokens;
      }
      admitted.push_back(t.sid);
    }
    for (const Task& t : ordered) {
      if (t.sid == primary) continue;
      auto sit = sessions_.find(t.sid);
      if (sit == sessions_.end() || sit->second.complete) {
        admitted.push_back(t.sid);  // stale task: drop it from the queue
        continue;
      }
      SessionInfo& s = sit->second;
      if (have_class) {
        const bool class_strict = (mode == THROUGHPUT_FIRST || mode == LATENCY_FIRST);
        if (class_strict && s.class_key != cls) {
          ++d_guard;
          deferred.emplace_back(t.sid, t.epoch);
          continue;
        }
      } else {
        have_class = true;
        cls = s.class_key;
        mode = s.mode;
        ceiling = s.token_ceiling;
      }
      if (requires_bucket_cohesion(mode) && ceiling >= 0 && s.token_ceiling != ceiling) {
        ++d_guard;
        deferred.emplace_back(t.sid, t.epoch);
        continue;
      }
      const int64_t pmin = bmin < 0 ? s.kv_tokens : std::min(bmin, s.kv_tokens);
      const int64_t pmax = bmax < 0 ? s.kv_tokens : std::max(bmax, s.kv_tokens);
      if (!allows_skew(mode, pmin, pmax)) {
        ++d_guard;
        deferred.emplace_back(t.sid, t.epoch);
        continue;
      }
      const bool full = (int64_t)slots.size() >= max_batch;
      const bool kv_out = !slots.empty() && total + s.kv_tokens > max_total_kv;
      if (full || kv_out) {
        if (full)
          ++d_cap;
        else
          ++d_kv;
        deferred.emplace_back(t.sid, t.epoch);
        continue;
      }
      slots.emplace_back(t.sid, t.epoch, s.kv_tokens);
      bmin = pmin;
      bmax = pmax;
      total += s.kv_tokens;
      admitted.push_back(t.sid);
    }
    for (int64_t sid : admitted) remove(sid);
    py::dict d;
    d["slots"] = slots;
    d["deferred"] = deferred;
    d["total_kv_tokens"] = total;
    d["deferred_for_capacity"] = d_cap;
    d["deferred_for_kv_budget"] = d_kv;
    d["deferred_for_guardrail"] = d_guard;
    return d;
  }

 private:
  SessionInfo& get(int64_t sid) {
    auto it = sessions_.find(sid);
    if (it == sessions_.end()) throw std::out_of_range("unknown session " + std::to_string(sid));
    return it->second;
  }
  std::unordered_map<int64_t, SessionInfo> sessions_;
  std::set<Task> queue_;
  std::unordered_map<int64_t, Task> index_;
  int64_t next_epoch_ = 0;
};

// ------------------------------------------------------------------------------------------------
constexpr size_t kFrameHeader = 49;

py::bytes encode_frame_header(const std::string& collective_id16, uint32_t seq, uint32_t sender, uint32_t layer,
                              uint32_t step, uint32_t slot, uint32_t stream, uint32_t count, int lane) {
  if (collective_id16.size() != 16) throw std::invalid_argument("collective id must be 16 bytes");
  if (lane < 0 || lane > 4) throw std::invalid_argument("invalid collective lane tag");
  std::string b(kFrameHeader, '\0');
  std::copy(collective_id16.begin(), collective_id16.end(), b.begin());
  uint32_t vals[7] = {seq, sender, layer, step, slot, stream, count};
  size_t o = 16;
  for (uint32_t v : vals) {
    b[o++] = (char)((v >> 24) & 0xff);
    b[o++] = (char)((v >> 16) & 0xff);
    b[o++] = (char)((v >> 8) & 0xff);
    b[o++] = (char)(v & 0xff);
  }
  b[o] = (char)lane;
  return py::bytes(b);
}

py::tuple decode_frame_header(const std::string& b) {
  if (b.size() != kFrameHeader)
    throw std::invalid_argument("serving frame header size " + std::to_string(b.size()) + " did not match 49");
  uint32_t v[7];
  size_t o = 16;
  for (int i = 0; i < 7; ++i) {
    v[i] = ((uint32_t)(uint8_t)b[o] << 24) | ((uint32_t)(uint8_t)b[o + 1] << 16) | ((uint32_t)(uint8_t)b[o + 2] << 8) |
           (uint32_t)(uint8_t)b[o + 3];
    o += 4;
  }
  int lane = (uint8_t)b[o];
  if (lane > 4) throw std::invalid_argument("invalid collective lane tag " + std::to_string(lane));
  return py::make_tuple(py::bytes(b.substr(0, 16)), v[0], v[1], v[2], v[3], v[4], v[5], v[6], lane);
}

// ------------------------------------------------------------------------------------------------
// Ring all-reduce over n ranks: chunk indices this position sends and receives at step s
// (reduce-scatter: send (p - s) mod n, recv (p - s - 1) mod n; all-gather: send (p - s + 1) mod n,
// recv (p - s) mod n).
py::tuple ring_chunk_plan(int64_t position, int64_t n, int64_t step, bool all_gather) {
  auto md = [n](int64_t x) { return ((x % n) + n) % n; };
  if (!all_gather) return py::make_tuple(md(position - step), md(position - step - 1));
  return py::make_tuple(md(position - step + 1), md(position - step));
}

// [start, end) element ranges of n chunks of `len` elements, first chunks one longer.
std::vector<std::pair<int64_t, int64_t>> chunk_ranges(int64_t len, int64_t n) {
  std::vector<std::pair<int64_t, int64_t>> r;
  const int64_t per = (len + n - 1) / n;
  for (int64_t i = 0; i < n; ++i) {
    int64_t a = std::min(len, i * per), b = std::min(len, (i + 1) * per);
    r.emplace_back(a, b);
  }
  return r;
}

}  // namespace mesh_rt

PYBIND11_MODULE(_runtime, m) {
  using namespace mesh_rt;
  m.doc() = "mesh_b200 native host runtime";
  py::class_<PageAllocator>(m, "PageAllocator")
      .def(py::init<int64_t, int64_t>(), py::arg("num_pages"), py::arg("reserved") = 0)
      .def("alloc", &PageAllocator::alloc)
      .def("free", &PageAllocator::free)
      .def_property_readonly("num_free", &PageAllocator::num_free)
      .def_property_readonly("num_used", &PageAllocator::num_used)
      .def_property_readonly("capacity", &PageAllocator::capacity);
  py::class_<DecodeScheduler>(m, "DecodeScheduler")
      .def(py::init<>())
      .def("register_session", &DecodeScheduler::register_session, py::arg("sid"), py::arg("class_key") = 0,
           py::arg("kv_tokens") = 0, py::arg("token_ceiling") = -1, py::arg("mode") = (int)THROUGHPUT_FIRST)
      .def("update", &DecodeScheduler::update, py::arg("sid"), py::arg("kv_tokens"), py::arg("token_ceiling") = -1)
      .def("set_complete", &DecodeScheduler::set_complete)
      .def("served", &DecodeScheduler::served)
      .def("steps_served", &DecodeScheduler::steps_served)
      .def("enqueue", &DecodeScheduler::enqueue)
      .def("remove", &DecodeScheduler::remove)
      .def("drop", &DecodeScheduler::drop)
      .def("queued", &DecodeScheduler::queued)
      .def("__len__", &DecodeScheduler::queue_len)
      .def("build_batch", &DecodeScheduler::build_batch, py::arg("primary"), py::arg("max_batch"),
           py::arg("max_total_kv"));
  m.def("encode_frame_header", &encode_frame_header);
  m.def("decode_frame_header", &decode_frame_header);
  m.def("ring_chunk_plan", &ring_chunk_plan);
  m.def("chunk_ranges", &chunk_ranges);
  m.attr("FRAME_HEADER_BYTES") = (int)kFrameHeader;
  m.attr("FIT_FIRST") = (int)FIT_FIRST;
  m.attr("THROUGHPUT_FIRST") = (int)THROUGHPUT_FIRST;
  m.attr("LATENCY_FIRST") = (int)LATENCY_FIRST;
  m.attr("RESILIENT_EDGE") = (int)RESILIENT_EDGE;
}
