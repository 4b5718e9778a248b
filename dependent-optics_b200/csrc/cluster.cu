// cluster.cu — the staging plan of a Mixtral block stack on a cluster of
// B200s, in the crate's cluster.rs vocabulary: devices and links
// (`Device`, `Link`, `derive_links`, src/cluster.rs:33-56, 307-348), homes
// where parameters and residuals live (`Home`, :134-158), windows of work
// run on one device (`Window`, :222-250) with the hops that deliver their
// inputs and carry their outputs (`Hop`, `HopKind`, :170-193), the plan
// (`StagePlan`, :252-257), its check (`StagePlan::check`, :1881-1928),
// message routing (`route_message`, :350-398) and the error variants
// (`StageError`, :266-292).
//
// The crate's planner tiles every matrix so that it fits devices with small
// buffers.  A B200 holds a whole Mixtral-8x7B block (1.45e9 parameters,
// 2.9 GB in bf16) and its residual, so here a home is a whole block on one
// GPU and a window is one block lens applied to one micro-batch (Exec
// `DOP_EXEC_BLOCK`, forward or backward).  The blocks are cut into
// pipeline stages (PP = the largest divisor of both the layer count and the
// GPU count), the GPUs left over hold data-parallel replicas of the pipeline,
// and each stage runs the one-forward-one-backward schedule over its
// replica's micro-batches.  Stage s keeps up to PP - s micro-batches in
// flight, so each of its blocks has that many residual slots (tape homes).
// Activations travel forward and their adjoints backward as hops between
// the stages' devices; at the end an Sgd window on every parameter home
// takes the other replicas' adjoints of the same layer (the data-parallel
// reduction) and applies the update.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <deque>
#include <memory>
#include <string>
#include <vector>

#include "block.cuh"

namespace dop {
int set_last_error(int code, const char* msg);

namespace stage {

struct WinRec {
  dop_window w{};
  std::vector<int64_t> in, out;  // hop indices
  std::string name;
};

struct Plan {
  std::vector<dop_home> homes;
  std::vector<WinRec> windows;
  std::vector<dop_hop> hops;
  std::vector<int64_t> peak;  // per device
  int64_t n_devices = 0;
  int64_t param_elems = 0;    // elements of one copy of the stack's parameters
};

// The fabric implied by a device list (derive_links): CPUs form a fabric,
// GPU i attaches to CPU i mod #cpus and peers the GPUs on that CPU; with no
// CPU every GPU peers every other.
std::vector<dop_link> derive_links(const dop_device* dev, int64_t n) {
  std::vector<int> cpus, gpus;
  for (int64_t i = 0; i < n; ++i) (dev[i].kind == DOP_DEVICE_CPU ? cpus : gpus).push_back((int)i);
  std::vector<dop_link> links;
  auto all_pairs = [&](const std::vector<int>& g) {
    for (size_t i = 0; i < g.size(); ++i)
      for (size_t j = i + 1; j < g.size(); ++j) links.push_back(dop_link{g[i], g[j]});
  };
  all_pairs(cpus);
  if (cpus.empty()) {
    all_pairs(gpus);
  } else {
    std::vector<std::vector<int>> host(cpus.size());
    for (size_t i = 0; i < gpus.size(); ++i) {
      links.push_back(dop_link{gpus[i], cpus[i % cpus.size()]});
      host[i % cpus.size()].push_back(gpus[i]);
    }
    for (auto& g : host) all_pairs(g);
  }
  return links;
}

// Shortest path from `from` to `to` whose intermediate devices have `bytes`
// free (route_message); empty when there is none.
std::vector<int> route(const std::vector<dop_link>& links, const std::vector<int64_t>& free_b,
                       int from, int to, int64_t bytes) {
  const int n = (int)free_b.size();
  if (from == to || bytes == 0) return {from};
  if (from < 0 || to < 0 || from >= n || to >= n) return {};
  std::vector<std::vector<int>> nb(n);
  for (const auto& l : links)
    if (l.a >= 0 && l.b >= 0 && l.a < n && l.b < n && l.a != l.b) {
      nb[l.a].push_back(l.b);
      nb[l.b].push_back(l.a);
    }
  std::vector<int> prev(n, -1);
  std::deque<int> q;
  prev[from] = from;
  q.push_back(from);
  while (!q.empty()) {
    const int u = q.front();
    q.pop_front();
    if (u == to) break;
    for (int v : nb[u]) {
      if (prev[v] >= 0 || (v != to && free_b[v] < bytes)) continue;
      prev[v] = u;
      q.push_back(v);
    }
  }
  if (prev[to] < 0) return {};
  std::vector<int> path{to};
  for (int c = to; c != from; c = prev[c]) path.push_back(prev[c]);
  std::reverse(path.begin(), path.end());
  return path;
}

[[noreturn]] void stage_error(int code, const std::string& msg) { throw Error(code, msg); }

struct Item {       // one step of a stage's 1F1B program
  int pass;         // DOP_PASS_FWD / DOP_PASS_BWD
  int micro;        // index within the replica
};

Plan* stage_mixtral(const dop_mixtral_cfg& cfg, int64_t global_batch, int64_t seq,
                    int64_t micro_batches, int precision, const dop_device* dev, int64_t n_dev,
                    const dop_link* links_in, int64_t n_links) {
  DOP_REQUIRE(cfg.layers >= 1 && global_batch >= 1 && seq >= 1 && micro_batches >= 1,
              "layers, batch, seq and micro-batches must be >= 1");
  DOP_REQUIRE(global_batch % micro_batches == 0, "global batch must split into equal micro-batches");
  std::vector<int> gpus;
  for (int64_t i = 0; i < n_dev; ++i)
    if (dev[i].kind == DOP_DEVICE_GPU) gpus.push_back((int)i);
  if (gpus.empty()) stage_error(DOP_E_NO_DEVICE, "the cluster has no GPU");
  const int L = (int)cfg.layers, G = (int)gpus.size();
  int PP = 1;
  for (int p = std::min(L, G); p >= 1; --p)
    if (L % p == 0 && G % p == 0) { PP = p; break; }
  const int DP = G / PP, per_stage = L / PP;
  DOP_REQUIRE(micro_batches >= DP, "fewer micro-batches than data-parallel replicas");
  const int64_t mb = global_batch / micro_batches;  // sequences per micro-batch
  const LayerOffsets off = layer_offsets(cfg);
  const int64_t lp = off.total;                      // parameters of one block
  const int64_t pbytes = lp * ((precision == DOP_BF16 ? 2 : 4) + 4);  // weights + fp32 adjoint
  const int64_t tape = (int64_t)Block(cfg, mb, seq, precision, 0, 1, false).bytes;
  const int64_t act = mb * seq * cfg.dim * 4;        // one fp32 activation or adjoint
  std::vector<dop_link> links =
      n_links > 0 ? std::vector<dop_link>(links_in, links_in + n_links) : derive_links(dev, n_dev);

  // capacity checks (StageError variants)
  int64_t cap_total = 0, largest = 0;
  for (int g : gpus) {
    cap_total += dev[g].buffer_bytes;
    largest = std::max<int64_t>(largest, dev[g].buffer_bytes);
  }
  if ((__int128)pbytes * L > cap_total)
    stage_error(DOP_E_PARAMS_EXCEED_CLUSTER,
                "parameters need " + std::to_string((long long)(pbytes * L)) + " bytes, the GPUs hold " +
                    std::to_string((long long)cap_total));
  if (pbytes + tape + 2 * act > largest)
    stage_error(DOP_E_TILE_EXCEEDS_DEVICES,
                "one block with one micro-batch needs " + std::to_string((long long)(pbytes + tape + 2 * act)) +
                    " bytes, the largest GPU holds " + std::to_string((long long)largest));

  std::unique_ptr<Plan> plan(new Plan());
  plan->n_devices = n_dev;
  plan->param_elems = lp * L;
  plan->peak.assign(n_dev, 0);
  std::vector<int64_t> stored(n_dev, 0);
  const int Mr0 = (int)micro_batches;
  auto replica_micros = [&](int r) {  // global micro-batch indices of replica r
    std::vector<int> m;
    for (int g = r; g < Mr0; g += DP) m.push_back(g);
    return m;
  };
  auto device_of = [&](int r, int s) { return gpus[r * PP + s]; };
  auto slots_of = [&](int r, int s) {
    return std::max(1, std::min(PP - s, (int)replica_micros(r).size()));
  };
  // homes and the device budget
  for (int r = 0; r < DP; ++r)
    for (int s = 0; s < PP; ++s) {
      const int d = device_of(r, s), slots = slots_of(r, s);
      for (int l = s * per_stage; l < (s + 1) * per_stage; ++l) {
        dop_home h{};
        h.kind = DOP_HOME_PARAM; h.device = d; h.layer = l; h.replica = r; h.slot = -1;
        h.row_begin = 0; h.row_end = 1; h.col_begin = 0; h.col_end = lp; h.stride = lp;
        h.bytes = pbytes;
        plan->homes.push_back(h);
        stored[d] += pbytes;
        for (int k = 0; k < slots; ++k) {
          dop_home t{};
          t.kind = DOP_HOME_TAPE; t.device = d; t.layer = l; t.replica = r; t.slot = k;
          t.row_begin = 0; t.row_end = 1; t.col_begin = 0; t.col_end = tape; t.stride = tape;
          t.bytes = tape;
          plan->homes.push_back(t);
          stored[d] += tape;
        }
      }
      const int64_t need = stored[d] + 2 * slots * act;
      plan->peak[d] = need;
      if (need > dev[d].buffer_bytes) {
        const int64_t free_b = dev[d].buffer_bytes - (stored[d] - per_stage * slots * tape);
        stage_error(DOP_E_TAPE_EXCEEDS_CLUSTER,
                    "stage " + std::to_string(s) + " on " + dev[d].name + " needs " +
                        std::to_string((long long)need) + " bytes for " + std::to_string(slots) +
                        " micro-batches in flight; " + std::to_string((long long)free_b) +
                        " bytes are free after its parameters");
      }
    }
  std::vector<int64_t> free_b(n_dev);
  for (int64_t i = 0; i < n_dev; ++i) free_b[i] = std::max<int64_t>(0, dev[i].buffer_bytes - plan->peak[i]);

  // 1F1B programs per (replica, stage) and the global order
  std::vector<std::vector<Item>> prog(DP * PP);
  for (int r = 0; r < DP; ++r) {
    const int Mr = (int)replica_micros(r).size();
    for (int s = 0; s < PP; ++s) {
      auto& p = prog[r * PP + s];
      const int warm = std::min(PP - s - 1, Mr);
      int f = 0, b = 0;
      for (; f < warm; ++f) p.push_back({DOP_PASS_FWD, f});
      while (f < Mr) {
        p.push_back({DOP_PASS_FWD, f++});
        p.push_back({DOP_PASS_BWD, b++});
      }
      while (b < Mr) p.push_back({DOP_PASS_BWD, b++});
    }
  }
  // done[r][s][pass][m]
  std::vector<std::vector<char>> done(DP * PP * 2);
  for (int r = 0; r < DP; ++r)
    for (int s = 0; s < PP; ++s)
      for (int ps = 0; ps < 2; ++ps) done[(r * PP + s) * 2 + ps].assign(replica_micros(r).size(), 0);
  auto is_done = [&](int r, int s, int ps, int m) { return done[(r * PP + s) * 2 + ps][m] != 0; };

  // a message from (replica r, stage sf) to stage st: one hop per link of its route
  auto add_message = [&](int r, int sf, int st, int kind, int layer, int micro, int64_t& first,
                         int64_t& count) {
    const int a = device_of(r, sf), b = device_of(r, st);
    std::vector<int> path = route(links, free_b, a, b, act);
    if (path.empty())
      stage_error(DOP_E_ROUTE_UNAVAILABLE, "no route from " + std::string(dev[a].name) + " to " +
                                               dev[b].name + " for " + std::to_string((long long)act) +
                                               " bytes");
    first = (int64_t)plan->hops.size();
    for (size_t i = 0; i + 1 < path.size(); ++i) {
      dop_hop h{};
      h.from = path[i]; h.to = path[i + 1]; h.kind = kind; h.bytes = act;
      h.offset = 0; h.elems = act / 4; h.row_begin = 0; h.row_end = mb * seq;
      h.col_begin = 0; h.col_end = cfg.dim; h.stride = cfg.dim;
      h.layer = layer; h.micro = micro; h.replica = r;
      plan->hops.push_back(h);
    }
    count = (int64_t)plan->hops.size() - first;
  };

  std::vector<size_t> pc(DP * PP, 0);
  // the hops a stage's next window waits for, created by the producing window
  struct Waiting { int r, s, ps, m; std::vector<int64_t> hops; };
  std::vector<Waiting> waiting;
  size_t remaining = 0;
  for (auto& p : prog) remaining += p.size();
  {
    while (remaining > 0) {
      bool progressed = false;
      for (int r = 0; r < DP; ++r)
        for (int s = 0; s < PP; ++s) {
          auto& p = prog[r * PP + s];
          size_t& i = pc[r * PP + s];
          if (i >= p.size()) continue;
          const Item it = p[i];
          const bool ready = it.pass == DOP_PASS_FWD ? (s == 0 || is_done(r, s - 1, 0, it.micro))
                                                     : (s == PP - 1 ? is_done(r, s, 0, it.micro)
                                                                    : is_done(r, s + 1, 1, it.micro));
          if (!ready) continue;
          const int gm = replica_micros(r)[it.micro];
          const int slot = it.micro % slots_of(r, s);
          std::vector<int64_t> inbound;
          for (auto& wv : waiting)
            if (wv.r == r && wv.s == s && wv.ps == it.pass && wv.m == it.micro) inbound = wv.hops;
          // the stage's blocks, in pass order
          for (int k = 0; k < per_stage; ++k) {
            const int l = it.pass == DOP_PASS_FWD ? s * per_stage + k : (s + 1) * per_stage - 1 - k;
            WinRec w;
            w.w.device = device_of(r, s); w.w.pass = it.pass; w.w.exec = DOP_EXEC_BLOCK;
            w.w.layer = l; w.w.micro = gm; w.w.replica = r; w.w.slot = slot;
            w.w.batch_begin = gm * mb; w.w.batch_end = (gm + 1) * mb;
            w.w.tape_bytes = tape; w.w.param_bytes = pbytes; w.w.param_offset = (int64_t)l * lp;
            w.w.din = cfg.dim; w.w.dout = cfg.dim;
            w.w.resident_bytes = plan->peak[w.w.device];
            for (size_t h = 0; h < plan->homes.size(); ++h)
              if (plan->homes[h].kind == DOP_HOME_PARAM && plan->homes[h].layer == l &&
                  plan->homes[h].replica == r)
                w.w.home = (int32_t)h;
            char nm[96];
            snprintf(nm, sizeof nm, "%s.l%d.m%d.r%d", it.pass == DOP_PASS_FWD ? "fwd" : "bwd", l, gm, r);
            w.name = nm;
            if (k == 0) w.in = inbound;
            if (k == per_stage - 1) {  // the stage's result leaves for the neighbour stage
              const int to = it.pass == DOP_PASS_FWD ? s + 1 : s - 1;
              if (to >= 0 && to < PP) {
                int64_t first, count;
                add_message(r, s, to, it.pass == DOP_PASS_FWD ? DOP_HOP_ACTIVATION : DOP_HOP_ADJOINT,
                            l, gm, first, count);
                std::vector<int64_t> hs;
                for (int64_t h = first; h < first + count; ++h) hs.push_back(h);
                w.out = hs;
                waiting.push_back({r, to, it.pass, it.micro, hs});
              }
            }
            plan->windows.push_back(w);
          }
          done[(r * PP + s) * 2 + (it.pass == DOP_PASS_FWD ? 0 : 1)][it.micro] = 1;
          ++i;
          --remaining;
          progressed = true;
        }
      if (!progressed) throw Error(DOP_E_STATE, "pipeline schedule does not progress");
    }
    // data-parallel reduction and update: one Sgd window per parameter home,
    // taking the other replicas' adjoints of the same layer
    for (int l = 0; l < L; ++l) {
      const int s = l / per_stage;
      for (int r = 0; r < DP; ++r) {
        WinRec w;
        w.w.device = device_of(r, s); w.w.pass = DOP_PASS_BWD; w.w.exec = DOP_EXEC_SGD;
        w.w.layer = l; w.w.micro = -1; w.w.replica = r; w.w.slot = -1;
        w.w.param_bytes = pbytes; w.w.param_offset = (int64_t)l * lp; w.w.din = 1; w.w.dout = lp;
        w.w.resident_bytes = plan->peak[w.w.device];
        for (size_t h = 0; h < plan->homes.size(); ++h)
          if (plan->homes[h].kind == DOP_HOME_PARAM && plan->homes[h].layer == l &&
              plan->homes[h].replica == r)
            w.w.home = (int32_t)h;
        for (int o = 0; o < DP; ++o) {
          if (o == r) continue;
          dop_hop h{};
          h.from = device_of(o, s); h.to = device_of(r, s); h.kind = DOP_HOP_ADJOINT;
          h.bytes = lp * 4; h.elems = lp; h.row_begin = 0; h.row_end = 1; h.col_begin = 0;
          h.col_end = lp; h.stride = lp; h.layer = l; h.micro = -1; h.replica = o;
          w.in.push_back((int64_t)plan->hops.size());
          plan->hops.push_back(h);
        }
        char nm[64];
        snprintf(nm, sizeof nm, "sgd.l%d.r%d", l, r);
        w.name = nm;
        plan->windows.push_back(w);
      }
    }
  }
  for (auto& w : plan->windows) {
    w.w.n_inbound = (int32_t)w.in.size();
    w.w.n_outbound = (int32_t)w.out.size();
  }
  return plan.release();
}

// StagePlan::check: one copy of the parameters covered, device budgets kept.
void check(const Plan& p, const dop_device* dev, int64_t n_dev, int64_t param_elems) {
  int64_t covered = 0;
  for (const auto& h : p.homes)
    if (h.kind == DOP_HOME_PARAM && h.replica == 0) covered += (h.row_end - h.row_begin) * (h.col_end - h.col_begin);
  if (covered != param_elems)
    throw Error(DOP_E_INVALID, "parameter homes cover " + std::to_string((long long)covered) +
                                   " elements, the model has " + std::to_string((long long)param_elems));
  DOP_REQUIRE(n_dev == p.n_devices, "the plan was made for another device list");
  for (int64_t d = 0; d < n_dev; ++d) {
    int64_t stored = 0;
    for (const auto& h : p.homes)
      if (h.device == d) stored += h.bytes;
    if (stored > dev[d].buffer_bytes)
      throw Error(DOP_E_INVALID, std::string(dev[d].name) + " stores " + std::to_string((long long)stored) +
                                     " bytes with a buffer of " + std::to_string((long long)dev[d].buffer_bytes));
    if (p.peak[d] > dev[d].buffer_bytes)
      throw Error(DOP_E_INVALID, std::string(dev[d].name) + " peaks at " + std::to_string((long long)p.peak[d]) +
                                     " bytes with a buffer of " + std::to_string((long long)dev[d].buffer_bytes));
  }
  for (const auto& w : p.windows) {
    DOP_REQUIRE(w.w.device >= 0 && w.w.device < n_dev, "window on a device outside the cluster");
    if (w.w.resident_bytes > dev[w.w.device].buffer_bytes)
      throw Error(DOP_E_INVALID, "window " + w.name + " uses more than its device's buffer");
    for (int64_t h : w.in) DOP_REQUIRE(p.hops[h].to >= 0 && p.hops[h].to < n_dev, "hop outside the cluster");
  }
}

std::string trace(const Plan& p) {
  std::string t = "MEMBERS " + std::to_string((long long)p.n_devices) + "\n";
  for (int64_t r = 0; r < p.n_devices; ++r) t += "JOIN " + std::to_string((long long)r) + "\n";
  auto hop = [&](int64_t i) {
    const dop_hop& h = p.hops[i];
    t += "HOP " + std::to_string(h.from) + " " + std::to_string(h.to) + " " + std::to_string(h.kind) +
         " " + std::to_string((long long)h.bytes) + "\n";
  };
  for (const auto& w : p.windows) {
    for (int64_t h : w.in) hop(h);
    t += "COMPUTE " + std::to_string(w.w.device) + " " + std::to_string(w.w.exec) + " " +
         std::to_string(w.w.pass) + "\n";
    for (int64_t h : w.out) hop(h);
  }
  t += "DONE\n";
  return t;
}

}  // namespace stage
}  // namespace dop

struct dop_stage_plan {
  dop::stage::Plan* p;
};

#define DOP_STAGE_GUARD(...)                                     \
  try {                                                          \
    __VA_ARGS__;                                                 \
    return DOP_OK;                                               \
  } catch (const dop::Error& e) {                                \
    return dop::set_last_error(e.code, e.what());                \
  } catch (const std::bad_alloc&) {                              \
    return dop::set_last_error(DOP_E_NOMEM, "host allocation failed"); \
  } catch (const std::exception& e) {                            \
    return dop::set_last_error(DOP_E_INVALID, e.what());         \
  }

extern "C" {

int dop_derive_links(const dop_device* devices, int64_t n_devices, dop_link* out, int64_t cap,
                     int64_t* count) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(count && (devices || n_devices == 0) && (out || cap == 0), "null pointer");
    auto l = dop::stage::derive_links(devices, n_devices);
    *count = (int64_t)l.size();
    DOP_REQUIRE(!out || cap >= (int64_t)l.size(), "output capacity too small");
    for (size_t i = 0; out && i < l.size(); ++i) out[i] = l[i];
  })
}

int dop_route_message(const dop_link* links, int64_t n_links, const int64_t* free_bytes,
                      int64_t n_devices, int32_t from, int32_t to, int64_t bytes, int32_t* path,
                      int64_t cap, int64_t* len) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(len && free_bytes && (links || n_links == 0) && (path || cap == 0), "null pointer");
    std::vector<dop_link> l(links, links + n_links);
    std::vector<int64_t> f(free_bytes, free_bytes + n_devices);
    auto p = dop::stage::route(l, f, from, to, bytes);
    if (p.empty())
      throw dop::Error(DOP_E_ROUTE_UNAVAILABLE, "no route from " + std::to_string(from) + " to " +
                                                    std::to_string(to) + " for " +
                                                    std::to_string((long long)bytes) + " bytes");
    *len = (int64_t)p.size();
    DOP_REQUIRE(!path || cap >= (int64_t)p.size(), "output capacity too small");
    for (size_t i = 0; path && i < p.size(); ++i) path[i] = p[i];
  })
}

int dop_stage_mixtral(const dop_mixtral_cfg* cfg, int64_t global_batch, int64_t seq,
                      int64_t micro_batches, int precision, const dop_device* devices,
                      int64_t n_devices, const dop_link* links, int64_t n_links,
                      dop_stage_plan** out) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(cfg && out && (devices || n_devices == 0) && (links || n_links == 0), "null pointer");
    DOP_REQUIRE(precision == DOP_F32 || precision == DOP_BF16, "precision must be DOP_F32 or DOP_BF16");
    auto* p = dop::stage::stage_mixtral(*cfg, global_batch, seq, micro_batches, precision, devices,
                                        n_devices, links, n_links);
    *out = new dop_stage_plan{p};
  })
}

int dop_plan_destroy(dop_stage_plan* plan) {
  if (plan) {
    delete plan->p;
    delete plan;
  }
  return DOP_OK;
}

int64_t dop_plan_home_count(const dop_stage_plan* p) { return p ? (int64_t)p->p->homes.size() : -1; }
int64_t dop_plan_window_count(const dop_stage_plan* p) { return p ? (int64_t)p->p->windows.size() : -1; }
int64_t dop_plan_hop_count(const dop_stage_plan* p) { return p ? (int64_t)p->p->hops.size() : -1; }

int dop_plan_home(const dop_stage_plan* p, int64_t i, dop_home* out) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(p && out && i >= 0 && i < (int64_t)p->p->homes.size(), "bad home index");
    *out = p->p->homes[i];
  })
}

int dop_plan_window(const dop_stage_plan* p, int64_t i, dop_window* out) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(p && out && i >= 0 && i < (int64_t)p->p->windows.size(), "bad window index");
    *out = p->p->windows[i].w;
  })
}

int dop_plan_window_hop(const dop_stage_plan* p, int64_t i, int outbound, int64_t j,
                        int64_t* hop_index) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(p && hop_index && i >= 0 && i < (int64_t)p->p->windows.size(), "bad window index");
    const auto& v = outbound ? p->p->windows[i].out : p->p->windows[i].in;
    DOP_REQUIRE(j >= 0 && j < (int64_t)v.size(), "bad hop position");
    *hop_index = v[j];
  })
}

int dop_plan_hop(const dop_stage_plan* p, int64_t i, dop_hop* out) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(p && out && i >= 0 && i < (int64_t)p->p->hops.size(), "bad hop index");
    *out = p->p->hops[i];
  })
}

int dop_plan_check(const dop_stage_plan* p, const dop_device* devices, int64_t n_devices,
                   int64_t param_elems) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(p && devices, "null pointer");
    dop::stage::check(*p->p, devices, n_devices, param_elems);
  })
}

int dop_plan_trace(const dop_stage_plan* p, char* buf, int64_t cap, int64_t* len) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(p && len && (buf || cap == 0), "null pointer");
    const std::string t = dop::stage::trace(*p->p);
    *len = (int64_t)t.size();
    if (buf) {
      DOP_REQUIRE(cap > (int64_t)t.size(), "output capacity too small");
      std::memcpy(buf, t.c_str(), t.size() + 1);
    }
  })
}

int dop_run_window(dop_block* blk, const dop_window* w, const void* params, const float* in,
                   float* out, float* dparams, void* stream) {
  DOP_STAGE_GUARD({
    DOP_REQUIRE(blk && w && params && in && out, "null pointer");
    DOP_REQUIRE(w->exec == DOP_EXEC_BLOCK, "dop_run_window runs block windows");
    auto* b = reinterpret_cast<dop::Block*>(blk);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (w->pass == DOP_PASS_FWD) {
      b->forward(params, in, out, s);
    } else {
      DOP_REQUIRE(dparams, "a backward window needs dparams");
      b->backward(params, in, out, dparams, s);
    }
  })
}

}  // extern "C"
