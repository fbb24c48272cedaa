// pybind11 module kvbm_b200._kvbm_core: the CPU-side block-manager core.
//
// Sequence hashes cross the boundary as Python ints packed as
// position << 128 | parent << 64 | lineage. Calls that touch a pool release
// the GIL while they hold the pool's mutex.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "block_pool.hpp"
#include "branch_tracker.hpp"
#include "disk_pool.hpp"
#include "hash.hpp"
#include "registry.hpp"
#include "tinylfu.hpp"
#include "tracker.hpp"

namespace py = pybind11;
using namespace kvbm;

namespace {

py::int_ to_py(const SeqHash& h) {
  py::int_ pos(h.position), par(h.parent), lin(h.lineage);
  py::object r = (pos << py::int_(128)) | (par << py::int_(64)) | lin;
  return py::reinterpret_borrow<py::int_>(r);
}

SeqHash from_py(py::handle o) {
  SeqHash h;
  h.lineage = PyLong_AsUnsignedLongLongMask(o.ptr());
  py::object p = py::reinterpret_borrow<py::object>(o) >> py::int_(64);
  h.parent = PyLong_AsUnsignedLongLongMask(p.ptr());
  py::object q = py::reinterpret_borrow<py::object>(o) >> py::int_(128);
  h.position = static_cast<uint32_t>(PyLong_AsUnsignedLongLongMask(q.ptr()));
  if (PyErr_Occurred()) throw py::error_already_set();
  return h;
}

std::vector<SeqHash> from_py_list(const py::iterable& it) {
  std::vector<SeqHash> v;
  for (auto o : it) v.push_back(from_py(o));
  return v;
}

py::list to_py_list(const std::vector<SeqHash>& v) {
  py::list l;
  for (auto& h : v) l.append(to_py(h));
  return l;
}

// Hashes of the complete blocks of `tokens`, chained from `parent`.
py::list sequence_hashes(py::array_t<int32_t, py::array::c_style | py::array::forcecast> tokens, size_t block_size,
                         uint64_t salt, py::object parent) {
  if (block_size == 0) throw std::invalid_argument("block_size must be > 0");
  auto buf = tokens.request();
  const int32_t* p = static_cast<const int32_t*>(buf.ptr);
  const size_t n = static_cast<size_t>(buf.size) / block_size;
  std::vector<SeqHash> out;
  out.reserve(n);
  {
    std::optional<SeqHash> par;
    if (!parent.is_none()) par = from_py(parent);
    py::gil_scoped_release rel;
    const SeqHash* prev = par ? &*par : nullptr;
    for (size_t i = 0; i < n; ++i) {
      out.push_back(chain(prev, block_hash(p + i * block_size, block_size, salt), salt));
      prev = &out.back();
    }
  }
  return to_py_list(out);
}

}  // namespace

PYBIND11_MODULE(_kvbm_core, m) {
  m.doc() = "kvbm_b200 native block-manager core (C++20)";

  m.def("sequence_hashes", &sequence_hashes, py::arg("tokens"), py::arg("block_size"), py::arg("salt") = 0,
        py::arg("parent") = py::none());
  m.def("block_hash", [](py::array_t<int32_t, py::array::c_style | py::array::forcecast> t, uint64_t salt) {
    auto b = t.request();
    return block_hash(static_cast<const int32_t*>(b.ptr), static_cast<size_t>(b.size), salt);
  }, py::arg("tokens"), py::arg("salt") = 0);
  m.def("string_salt", &string_salt);
  m.def("hash_position", [](py::handle h) { return from_py(h).position; });
  m.def("hash_parent", [](py::handle h) { return from_py(h).parent; });
  m.def("hash_lineage", [](py::handle h) { return from_py(h).lineage; });
  m.def("make_hash", [](uint64_t lineage, uint64_t parent, uint32_t position) {
    SeqHash h;
    h.lineage = lineage;
    h.parent = parent;
    h.position = position;
    return to_py(h);
  });

  py::class_<TinyLfu, std::shared_ptr<TinyLfu>>(m, "TinyLfu")
      .def(py::init<size_t>(), py::arg("capacity") = (1u << 21))
      .def("touch", &TinyLfu::touch)
      .def("estimate", &TinyLfu::estimate)
      .def("size", &TinyLfu::size);

  py::class_<EventQueue, std::shared_ptr<EventQueue>>(m, "EventQueue")
      .def(py::init([](bool all, uint64_t min_pos, uint64_t max_pos) {
             EventPolicy p;
             p.all = all;
             p.min_pos = min_pos;
             p.max_pos = max_pos;
             return std::make_shared<EventQueue>(p);
           }),
           py::arg("all_events") = true, py::arg("min_position") = 16, py::arg("max_position") = 65536)
      .def("set_policy", [](EventQueue& q, bool all, uint64_t mn, uint64_t mx) {
        EventPolicy p;
        p.all = all;
        p.min_pos = mn;
        p.max_pos = mx;
        q.set_policy(p);
      })
      .def("set_enabled", &EventQueue::set_enabled)
      .def("pending", &EventQueue::pending)
      .def("drain", [](EventQueue& q) {
        py::list out;
        for (auto& e : q.drain()) out.append(py::make_tuple(e.kind == EventKind::Create ? "create" : "remove", to_py(e.hash)));
        return out;
      })
      .def("drain_batches", [](EventQueue& q, size_t max_batch) {
        py::list out;
        for (auto& [k, v] : q.drain_batches(max_batch))
          out.append(py::make_tuple(k == EventKind::Create ? "create" : "remove", to_py_list(v)));
        return out;
      }, py::arg("max_batch") = 1024);

  auto record = [](const BranchRecord& r) {
    py::dict d;
    d["position"] = r.position;
    d["fragment"] = r.fragment;
    d["current_fanout"] = r.current_fanout;
    d["max_fanout"] = r.max_fanout;
    d["observation_count"] = r.observations;
    d["last_updated_tick"] = r.last_tick;
    return d;
  };
  py::class_<BranchTracker, std::shared_ptr<BranchTracker>>(m, "BranchTracker")
      .def(py::init<size_t>(), py::arg("history_capacity") = 1024)
      .def("on_block_registered", [](BranchTracker& t, py::handle h) { t.on_registered(from_py(h)); })
      .def("is_branch_point", &BranchTracker::is_branch_point, py::arg("position"), py::arg("fragment"))
      .def("current_fanout", &BranchTracker::current_fanout, py::arg("position"), py::arg("fragment"))
      .def("current_branch_points", &BranchTracker::current_branch_points)
      .def("hot_branch_points", [record](const BranchTracker& t, size_t limit) {
        py::list out;
        for (auto& r : t.hot_branch_points(limit)) out.append(record(r));
        return out;
      }, py::arg("limit"))
      .def("branch_points_on_prefix", [record](const BranchTracker& t, py::iterable hs) {
        auto v = from_py_list(hs);
        py::list out;
        for (auto& r : t.on_prefix(v)) out.append(record(r));
        return out;
      })
      .def("branch_point_count", &BranchTracker::branch_point_count)
      .def("tracked_parent_count", &BranchTracker::tracked_parent_count)
      .def("history_len", &BranchTracker::history_len)
      .def_property_readonly("tick", &BranchTracker::tick);

  py::class_<Registry, std::shared_ptr<Registry>>(m, "Registry")
      .def(py::init([](std::shared_ptr<EventQueue> ev, std::shared_ptr<TinyLfu> f, std::shared_ptr<BranchTracker> b) {
             auto r = std::make_shared<Registry>(ev, f);
             if (b) r->set_branch_tracker(std::move(b));
             return r;
           }),
           py::arg("events") = nullptr, py::arg("frequency") = nullptr, py::arg("branch_tracker") = nullptr)
      .def("mark_present", [](Registry& r, py::handle h, int t) { r.mark_present(from_py(h), t); })
      .def("mark_absent", [](Registry& r, py::handle h, int t) { r.mark_absent(from_py(h), t); })
      .def("is_present", [](Registry& r, py::handle h, int t) { return r.is_present(from_py(h), t); },
           py::arg("hash"), py::arg("tier") = -1)
      .def("presence_mask", [](Registry& r, py::handle h) { return r.presence_mask(from_py(h)); })
      .def("check_presence", [](Registry& r, py::iterable hs, int t) {
        std::vector<bool> out;
        for (auto& h : from_py_list(hs)) out.push_back(r.is_present(h, t));
        return out;
      }, py::arg("hashes"), py::arg("tier") = -1)
      .def("touch", [](Registry& r, py::handle h) { r.touch(from_py(h)); })
      .def("frequency", [](Registry& r, py::handle h) { return r.frequency(from_py(h)); })
      .def("size", &Registry::size)
      .def_property_readonly("events", &Registry::events)
      .def_property_readonly("branch_tracker", &Registry::branch_tracker);

  py::enum_<SlotState>(m, "SlotState")
      .value("Reset", SlotState::Reset)
      .value("Mutable", SlotState::Mutable)
      .value("Staged", SlotState::Staged)
      .value("Primary", SlotState::Primary)
      .value("Duplicate", SlotState::Duplicate)
      .value("Inactive", SlotState::Inactive);

  py::class_<BlockPool, std::shared_ptr<BlockPool>>(m, "BlockPool")
      .def(py::init([](size_t n, size_t bs, const std::string& inactive, int tier, std::shared_ptr<Registry> reg,
                       const std::string& dup) {
             DupPolicy p = dup == "reject" ? DupPolicy::Reject : DupPolicy::Allow;
             if (dup != "reject" && dup != "allow") throw std::invalid_argument("duplicate_policy: allow|reject");
             return std::make_shared<BlockPool>(n, bs, inactive, tier, reg, p);
           }),
           py::arg("num_blocks"), py::arg("block_size") = 16, py::arg("inactive") = "lru", py::arg("tier") = 1,
           py::arg("registry") = nullptr, py::arg("duplicate_policy") = "allow")
      .def("allocate", [](BlockPool& p, size_t n) -> py::object {
        std::vector<SeqHash> ev;
        std::optional<std::vector<BlockId>> ids;
        {
          py::gil_scoped_release rel;
          ids = p.allocate(n, &ev);
        }
        if (!ids) return py::none();
        return py::make_tuple(*ids, to_py_list(ev));
      })
      .def("release_mutable", &BlockPool::release_mutable, py::call_guard<py::gil_scoped_release>())
      .def("release_mutable_many", [](BlockPool& p, const std::vector<BlockId>& ids) {
        py::gil_scoped_release rel;
        for (auto id : ids) p.release_mutable(id);
      })
      .def("stage", [](BlockPool& p, BlockId id, py::handle h) { p.stage(id, from_py(h)); })
      .def("unstage", &BlockPool::unstage)
      .def("release_staged", &BlockPool::release_staged)
      .def("register", [](BlockPool& p, BlockId id) {
        RegisterResult r;
        {
          py::gil_scoped_release rel;
          r = p.register_block(id);
        }
        return py::make_tuple(r.block_id, r.kind);
      })
      .def("stage_and_register", [](BlockPool& p, const std::vector<BlockId>& ids, py::iterable hashes) {
        auto hs = from_py_list(hashes);
        if (hs.size() != ids.size()) throw std::invalid_argument("ids and hashes differ in length");
        std::vector<std::pair<BlockId, int>> out;
        {
          py::gil_scoped_release rel;
          for (size_t i = 0; i < ids.size(); ++i) {
            p.stage(ids[i], hs[i]);
            auto r = p.register_block(ids[i]);
            out.emplace_back(r.block_id, r.kind);
          }
        }
        return out;
      })
      .def("match_prefix", [](BlockPool& p, py::iterable hashes) {
        auto hs = from_py_list(hashes);
        py::gil_scoped_release rel;
        return p.match_prefix(hs);
      })
      .def("scan", [](BlockPool& p, py::iterable hashes, bool touch) {
        auto hs = from_py_list(hashes);
        std::vector<std::pair<SeqHash, BlockId>> r;
        {
          py::gil_scoped_release rel;
          r = p.scan(hs, touch);
        }
        py::dict d;
        for (auto& [h, id] : r) d[to_py(h)] = id;
        return d;
      }, py::arg("hashes"), py::arg("touch") = false)
      .def("count_prefix", [](BlockPool& p, py::iterable hashes) { return p.count_prefix(from_py_list(hashes)); })
      .def("contains", [](BlockPool& p, py::handle h) { return p.contains(from_py(h)); })
      .def("add_ref", &BlockPool::add_ref)
      .def("release", &BlockPool::release, py::call_guard<py::gil_scoped_release>())
      .def("release_many", [](BlockPool& p, const std::vector<BlockId>& ids) {
        py::gil_scoped_release rel;
        for (auto id : ids) p.release(id);
      })
      .def("set_reset_on_release", &BlockPool::set_reset_on_release)
      .def("reset_inactive", &BlockPool::reset_inactive, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("total_blocks", &BlockPool::total_blocks)
      .def_property_readonly("block_size", &BlockPool::block_size)
      .def_property_readonly("tier", &BlockPool::tier)
      .def_property_readonly("inactive_kind", &BlockPool::inactive_kind)
      .def("reset_len", &BlockPool::reset_len)
      .def("inactive_len", &BlockPool::inactive_len)
      .def("available", &BlockPool::available)
      .def("active_len", &BlockPool::active_len)
      .def("state", &BlockPool::state)
      .def("refs", &BlockPool::refs)
      .def("hash_of", [](BlockPool& p, BlockId id) { return to_py(p.hash_of(id)); })
      .def_property_readonly("registry", &BlockPool::registry)
      .def("metrics", [](BlockPool& p) {
        const auto& m = p.metrics();
        py::dict d;
        d["allocations"] = m.allocations.load();
        d["allocations_from_reset"] = m.allocations_from_reset.load();
        d["evictions"] = m.evictions.load();
        d["registrations"] = m.registrations.load();
        d["registration_dedup"] = m.registration_dedup.load();
        d["duplicate_blocks"] = m.duplicate_blocks.load();
        d["match_hashes_requested"] = m.match_hashes_requested.load();
        d["match_blocks_returned"] = m.match_blocks_returned.load();
        d["scan_hashes_requested"] = m.scan_hashes_requested.load();
        d["scan_blocks_returned"] = m.scan_blocks_returned.load();
        d["allocate_failures"] = m.allocate_failures.load();
        return d;
      });

  py::class_<ConsolidatorTracker>(m, "ConsolidatorTracker")
      .def(py::init<>())
      .def("handle_store", [](ConsolidatorTracker& t, int src, const std::string& ext, std::optional<std::string> parent,
                              const std::vector<int32_t>& tokens, int64_t block_size, const std::string& lora) {
        return t.handle_store(src, ext, parent, tokens, block_size, lora);
      }, py::arg("source"), py::arg("external_hash"), py::arg("parent_external_hash"), py::arg("token_ids"),
         py::arg("block_size"), py::arg("lora_name") = "")
      .def("handle_remove", &ConsolidatorTracker::handle_remove)
      .def("handle_kvbm_store", [](ConsolidatorTracker& t, py::handle h) { return t.handle_kvbm_store(from_py(h)); })
      .def("handle_kvbm_remove", [](ConsolidatorTracker& t, py::handle h) { return t.handle_kvbm_remove(from_py(h)); })
      .def("handle_clear_all", &ConsolidatorTracker::handle_clear_all)
      .def("is_live", [](ConsolidatorTracker& t, py::handle h) { return t.is_live(from_py(h)); })
      .def("num_blocks", &ConsolidatorTracker::num_blocks)
      .def("num_external_mappings", &ConsolidatorTracker::num_external)
      .def("drain_events", [](ConsolidatorTracker& t) {
        py::list out;
        for (auto& e : t.drain()) {
          py::dict d;
          d["kind"] = e.kind == 0 ? "store" : (e.kind == 1 ? "remove" : "clear_all");
          if (e.kind != 2) {
            d["seq_hash"] = to_py(e.hash);
            d["router_hash"] = e.hash.lineage;
          }
          if (e.kind == 0) {
            d["token_ids"] = e.tokens;
            d["block_size"] = e.block_size;
            d["lora_name"] = e.lora.empty() ? py::object(py::none()) : py::object(py::str(e.lora));
          }
          d["source"] = e.source;
          out.append(d);
        }
        return out;
      });

  py::class_<PositionalIndex, std::shared_ptr<PositionalIndex>>(m, "PositionalIndex")
      .def(py::init<uint64_t, uint64_t>(), py::arg("max_seq_len"), py::arg("block_size"))
      .def("grow_to_max_seq_len", &PositionalIndex::grow_to)
      .def("apply", [](PositionalIndex& ix, py::int_ instance, const std::string& kind, py::iterable hashes) {
        const uint64_t lo = PyLong_AsUnsignedLongLongMask(instance.ptr());
        py::object hi_o = py::reinterpret_borrow<py::object>(instance) >> py::int_(64);
        const uint64_t hi = PyLong_AsUnsignedLongLongMask(hi_o.ptr());
        auto hs = from_py_list(hashes);
        if (kind == "create")
          ix.apply_create({hi, lo}, hs);
        else if (kind == "remove")
          ix.apply_remove({hi, lo}, hs);
        else
          throw std::invalid_argument("kind must be create|remove");
      })
      .def("remove_instance", [](PositionalIndex& ix, py::int_ instance) {
        const uint64_t lo = PyLong_AsUnsignedLongLongMask(instance.ptr());
        py::object hi_o = py::reinterpret_borrow<py::object>(instance) >> py::int_(64);
        ix.remove_instance({PyLong_AsUnsignedLongLongMask(hi_o.ptr()), lo});
      })
      .def("query_holders", [](PositionalIndex& ix, py::iterable hashes) -> py::object {
        auto r = ix.query(from_py_list(hashes));
        if (!r) return py::none();
        py::list insts;
        for (auto& [hi, lo] : r->second) insts.append((py::int_(hi) << py::int_(64)) | py::int_(lo));
        return py::make_tuple(to_py(r->first), insts);
      })
      .def("by_position", [](PositionalIndex& ix, uint64_t position) {
        py::list out;
        for (auto& [lin, insts] : ix.at_position(position)) {
          py::list holders;
          for (auto& [hi, lo] : insts) holders.append((py::int_(hi) << py::int_(64)) | py::int_(lo));
          out.append(py::make_tuple(py::int_(lin), holders));
        }
        return out;
      })
      .def("num_positions", &PositionalIndex::num_positions)
      .def("dropped_out_of_range", &PositionalIndex::dropped)
      .def("num_entries", &PositionalIndex::num_entries);

  py::register_exception<LockOrderError>(m, "LockOrderError", PyExc_RuntimeError);
  m.def("lock_check_enabled", &lock_check_enabled);
  // Takes a BlockPool-rank mutex, then a Registry-rank one: must raise
  // LockOrderError when checking is on (the registry ranks below the pool).
  m.def("lock_order_selftest", []() {
    RankedMutex pool(kRankBlockPool, "BlockPool"), reg(kRankRegistry, "Registry");
    std::lock_guard<RankedMutex> a(pool);
    std::lock_guard<RankedMutex> b(reg);
    return RankedMutex::held().size();
  });

  py::class_<DiskPool, std::shared_ptr<DiskPool>>(m, "DiskPool")
      .def(py::init<const std::string&, uint64_t, uint64_t, bool, bool, int>(), py::arg("path"),
           py::arg("num_blocks"), py::arg("block_bytes"), py::arg("direct") = false, py::arg("persistent") = false,
           py::arg("threads") = 4)
      .def("write", &DiskPool::write, py::call_guard<py::gil_scoped_release>())
      .def("read", &DiskPool::read, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("num_blocks", &DiskPool::num_blocks)
      .def_property_readonly("block_bytes", &DiskPool::block_bytes)
      .def_property_readonly("fd", &DiskPool::fd)
      .def_property_readonly("fd_direct", &DiskPool::fd_direct)
      .def_property_readonly("direct", &DiskPool::direct)
      .def_property_readonly("persistent", &DiskPool::persistent)
      .def_property_readonly("path", &DiskPool::path)
      .def("bytes_written", &DiskPool::bytes_written)
      .def("bytes_read", &DiskPool::bytes_read);
}
