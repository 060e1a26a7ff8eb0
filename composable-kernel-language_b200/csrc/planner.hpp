// Dependency inference, transitive reduction and temporary-storage planning for CKL programs.
//
// Pure C++17, no CUDA.  The rules restate the reference's analysis:
//   * conflict rule  - two accesses conflict unless both only read
//                      (lib/Core/MemoryEffects.cpp:51-54);
//   * alias rule     - the same base resource must-alias; a compiler allocation aliases
//                      nothing else; two distinct caller buffers may alias
//                      (lib/Core/MemoryEffects.cpp:89-97).  A plan compiled for bindings that
//                      are checked disjoint at bind time may treat distinct caller buffers as
//                      not aliasing (`externalsDisjoint`);
//   * regions        - must-alias accesses to provably disjoint byte intervals do not conflict,
//                      unless one of them is an allocation or free
//                      (lib/Analysis/GraphAnalysis.cpp:460-491);
//   * SSA edges      - a dispatch depends on the allocation node of each temporary it names
//                      (GraphAnalysis.cpp:449-456);
//   * reduction      - dispatch predecessors are kept only when no other dispatch lies on a
//                      path between them (lib/Analysis/GraphAlgorithms.cpp:10-46);
//   * memory plan    - a temporary joins an existing storage slot only when its whole use set
//                      is strictly ordered (by graph reachability) before or after every resident
//                      of that slot; best fit by least growth; slots pack into one heap per
//                      device and address space (lib/Core/MemoryPlanner.cpp:98-204).
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <limits>
#include <map>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace ckl::planning {

using NodeId = std::size_t;
using ResourceId = std::size_t;

enum Access : unsigned { Read = 1u, Write = 2u, Allocate = 4u, Free = 8u };

inline bool conflicting(unsigned lhs, unsigned rhs) {
  constexpr unsigned mutating = Write | Allocate | Free;
  return ((lhs | rhs) & mutating) != 0;
}

// Byte region of one access: whole buffer, unknown, or [offset, offset + length).
struct Region {
  enum Kind { Whole, Unknown, Interval } kind = Whole;
  std::int64_t offset = 0;
  std::int64_t length = 0;
  static bool disjoint(const Region &a, const Region &b) {
    return a.kind == Interval && b.kind == Interval &&
           (a.offset + a.length <= b.offset || b.offset + b.length <= a.offset);
  }
};

struct BoundAccess {
  ResourceId resource;
  unsigned bits;
  Region region;
};

enum class NodeKind { Dispatch, Alloc, Free };

struct GraphNode {
  NodeKind kind = NodeKind::Dispatch;
  bool unknown = false;
  std::vector<BoundAccess> accesses;
};

struct ProgramResource {
  bool temporary = false;  // a compiler allocation: a fresh identity
  bool persistent = false; // with `temporary`: dedicated storage, never shared
  int device = 0;
  std::size_t bytes = 0;
  std::size_t alignment = 256;
};

struct GraphEdge {
  NodeId from;
  NodeId to;
};

// ---------------------------------------------------------------------------------------
// Reachability (transitive closure) over a DAG given in any edge order.
class Reachability {
public:
  Reachability(std::size_t nodes, const std::vector<GraphEdge> &edges) : n_(nodes) {
    if (nodes && nodes > std::numeric_limits<std::size_t>::max() / nodes)
      throw std::overflow_error("memory-planning graph is too large");
    bits_.assign(n_ * n_, false);
    for (const GraphEdge &e : edges) {
      if (e.from >= n_ || e.to >= n_)
        throw std::out_of_range("memory-planning edge references an unknown graph node");
      if (e.from == e.to)
        throw std::invalid_argument("memory-planning graph contains a self edge");
      bits_[e.from * n_ + e.to] = true;
    }
    for (std::size_t via = 0; via < n_; ++via)
      for (std::size_t a = 0; a < n_; ++a) {
        if (!bits_[a * n_ + via])
          continue;
        for (std::size_t b = 0; b < n_; ++b)
          if (bits_[via * n_ + b])
            bits_[a * n_ + b] = true;
      }
    for (std::size_t a = 0; a < n_; ++a)
      if (bits_[a * n_ + a])
        throw std::invalid_argument("memory-planning graph must be acyclic");
  }
  bool operator()(NodeId from, NodeId to) const { return bits_[from * n_ + to]; }
  std::size_t size() const { return n_; }

private:
  std::size_t n_;
  std::vector<bool> bits_;
};

// ---------------------------------------------------------------------------------------
// Memory planner
enum class ResourceKind { Temporary, Persistent, External };

struct PlannerResource {
  std::string name;
  std::size_t bytes = 0;
  std::size_t alignment = 1;
  std::string addressSpace = "global";
  int device = 0;
  ResourceKind kind = ResourceKind::Temporary;
  std::vector<NodeId> users;
};

struct Heap {
  int device = 0;
  std::string addressSpace;
  std::size_t bytes = 0;
  std::size_t alignment = 1;
};

struct Assignment {
  ResourceId resource = 0;
  std::size_t heap = 0;
  std::size_t offset = 0;
  std::size_t bytes = 0;
  std::size_t slot = 0;
};

struct ReuseDecision {
  ResourceId resource = 0;
  std::size_t slot = 0;
  std::vector<ResourceId> sharesWith;
  std::string reason;
};

struct MemoryPlan {
  std::size_t baselineBytes = 0;
  std::size_t plannedBytes = 0;
  std::vector<Heap> heaps;
  std::vector<Assignment> assignments;
  std::vector<ReuseDecision> decisions;
  const Assignment *find(ResourceId id) const {
    for (const Assignment &a : assignments)
      if (a.resource == id)
        return &a;
    return nullptr;
  }
};

inline std::size_t roundUp(std::size_t value, std::size_t alignment) {
  if (!alignment || (alignment & (alignment - 1)))
    throw std::invalid_argument("resource alignment must be a nonzero power of two");
  if (value > std::numeric_limits<std::size_t>::max() - (alignment - 1))
    throw std::overflow_error("memory plan size overflow");
  return (value + alignment - 1) & ~(alignment - 1);
}

class MemoryPlanner {
public:
  explicit MemoryPlanner(bool reuse = true) : reuse_(reuse) {}

  MemoryPlan plan(std::size_t nodeCount, const std::vector<GraphEdge> &edges,
                  const std::vector<PlannerResource> &resources) const {
    Reachability reach(nodeCount, edges);
    // `first` strictly precedes `second` when every use of one reaches every use of the other.
    auto ordered = [&](const PlannerResource &first, const PlannerResource &second) {
      if (first.users.empty() || second.users.empty())
        return false;
      for (NodeId a : first.users)
        for (NodeId b : second.users)
          if (a == b || !reach(a, b))
            return false;
      return true;
    };
    struct Slot {
      int device;
      std::string space;
      std::size_t bytes, alignment;
      bool recyclable;
      std::vector<ResourceId> residents;
      std::size_t heap = 0, offset = 0;
    };
    std::vector<Slot> slots;
    std::vector<std::size_t> slotOf(resources.size(), SIZE_MAX);
    MemoryPlan out;
    for (ResourceId id = 0; id < resources.size(); ++id) {
      const PlannerResource &r = resources[id];
      if (!r.bytes)
        throw std::invalid_argument("memory-planning resource size must be nonzero");
      roundUp(r.bytes, r.alignment);
      for (NodeId user : r.users)
        if (user >= nodeCount)
          throw std::out_of_range("memory-planning resource references an unknown graph node");
      if (r.kind == ResourceKind::Temporary && r.users.empty())
        throw std::invalid_argument("temporary memory-planning resource must have at least one user");
      if (r.kind == ResourceKind::External)
        continue;
      std::size_t dedicated = roundUp(r.bytes, r.alignment);
      if (out.baselineBytes > std::numeric_limits<std::size_t>::max() - dedicated)
        throw std::overflow_error("memory plan baseline size overflow");
      out.baselineBytes += dedicated;
      std::size_t chosen = SIZE_MAX, bestGrowth = SIZE_MAX;
      if (reuse_ && r.kind == ResourceKind::Temporary) {
        for (std::size_t s = 0; s < slots.size(); ++s) {
          const Slot &slot = slots[s];
          if (!slot.recyclable || slot.device != r.device || slot.space != r.addressSpace)
            continue;
          bool fits = std::all_of(slot.residents.begin(), slot.residents.end(), [&](ResourceId o) {
            return ordered(r, resources[o]) || ordered(resources[o], r);
          });
          if (!fits)
            continue;
          std::size_t growth = std::max(slot.bytes, r.bytes) - slot.bytes;
          if (growth < bestGrowth) {
            chosen = s;
            bestGrowth = growth;
          }
        }
      }
      if (chosen == SIZE_MAX) {
        chosen = slots.size();
        slots.push_back({r.device, r.addressSpace, r.bytes, r.alignment,
                         r.kind == ResourceKind::Temporary, {}, 0, 0});
      }
      Slot &slot = slots[chosen];
      std::vector<ResourceId> before = slot.residents;
      slot.bytes = std::max(slot.bytes, r.bytes);
      slot.alignment = std::max(slot.alignment, r.alignment);
      slot.residents.push_back(id);
      slotOf[id] = chosen;
      std::string reason;
      if (!before.empty())
        reason = "all resource uses are ordered by existing graph edges";
      else if (r.kind == ResourceKind::Persistent)
        reason = "persistent resource gets dedicated storage";
      else
        reason = reuse_ ? "no compatible ordered lifetime" : "storage reuse disabled";
      out.decisions.push_back({id, chosen, std::move(before), std::move(reason)});
    }
    for (Slot &slot : slots) {
      auto heap = std::find_if(out.heaps.begin(), out.heaps.end(), [&](const Heap &h) {
        return h.device == slot.device && h.addressSpace == slot.space;
      });
      if (heap == out.heaps.end()) {
        out.heaps.push_back({slot.device, slot.space, 0, slot.alignment});
        heap = out.heaps.end() - 1;
      }
      slot.heap = static_cast<std::size_t>(heap - out.heaps.begin());
      heap->alignment = std::max(heap->alignment, slot.alignment);
      slot.offset = roundUp(heap->bytes, slot.alignment);
      if (slot.offset > std::numeric_limits<std::size_t>::max() - slot.bytes)
        throw std::overflow_error("memory plan heap size overflow");
      heap->bytes = slot.offset + slot.bytes;
    }
    for (Heap &h : out.heaps) {
      h.bytes = roundUp(h.bytes, h.alignment);
      if (out.plannedBytes > std::numeric_limits<std::size_t>::max() - h.bytes)
        throw std::overflow_error("memory plan total size overflow");
      out.plannedBytes += h.bytes;
    }
    for (ResourceId id = 0; id < resources.size(); ++id) {
      if (resources[id].kind == ResourceKind::External)
        continue;
      const Slot &slot = slots[slotOf[id]];
      out.assignments.push_back({id, slot.heap, slot.offset, resources[id].bytes, slotOf[id]});
    }
    return out;
  }

private:
  bool reuse_;
};

// ---------------------------------------------------------------------------------------
// Graph inference over one traced program.
struct ProgramGraph {
  std::vector<GraphEdge> edges;                       // all inferred edges, sorted, unique
  std::map<NodeId, std::vector<NodeId>> dependencies; // reduced dispatch predecessors
  std::vector<ResourceId> resourceOrder;              // first-access order over dispatches
  std::vector<std::vector<NodeId>> users;             // per program resource
  MemoryPlan memory;                                  // over temporaries, by resourceOrder
  std::vector<ResourceId> plannerToProgram;           // planner resource -> program resource
};

inline ProgramGraph inferGraph(const std::vector<GraphNode> &nodes,
                               const std::vector<ProgramResource> &resources, bool reuseStorage,
                               bool externalsDisjoint) {
  const std::size_t n = nodes.size();
  for (const GraphNode &node : nodes)
    for (const BoundAccess &a : node.accesses)
      if (a.resource >= resources.size())
        throw std::out_of_range("graph access references an unknown resource");
  std::map<std::pair<NodeId, NodeId>, int> edgeSet;
  auto add = [&](NodeId from, NodeId to) {
    if (from != to)
      edgeSet[{from, to}] = 1;
  };
  enum Alias { NoAlias, MayAlias, MustAlias };
  auto alias = [&](ResourceId a, ResourceId b) {
    if (a == b)
      return MustAlias;
    if (resources[a].temporary || resources[b].temporary || externalsDisjoint)
      return NoAlias;
    return MayAlias;
  };
  // SSA edges: allocation node -> dispatch naming that temporary.
  std::vector<NodeId> allocNode(resources.size(), SIZE_MAX);
  for (NodeId id = 0; id < n; ++id)
    if (nodes[id].kind == NodeKind::Alloc)
      for (const BoundAccess &a : nodes[id].accesses)
        allocNode[a.resource] = id;
  for (NodeId to = 0; to < n; ++to)
    if (nodes[to].kind == NodeKind::Dispatch)
      for (const BoundAccess &a : nodes[to].accesses)
        if (allocNode[a.resource] != SIZE_MAX && allocNode[a.resource] < to)
          add(allocNode[a.resource], to);
  // Memory, lifetime and unknown-effect barrier edges.
  for (NodeId from = 0; from < n; ++from)
    for (NodeId to = from + 1; to < n; ++to) {
      if (nodes[from].unknown || nodes[to].unknown) {
        add(from, to);
        continue;
      }
      for (const BoundAccess &lhs : nodes[from].accesses) {
        bool linked = false;
        for (const BoundAccess &rhs : nodes[to].accesses) {
          Alias rel = alias(lhs.resource, rhs.resource);
          if (rel == NoAlias || !conflicting(lhs.bits, rhs.bits))
            continue;
          bool lifetime = ((lhs.bits | rhs.bits) & (Allocate | Free)) != 0;
          if (!lifetime && rel == MustAlias && Region::disjoint(lhs.region, rhs.region))
            continue;
          add(from, to);
          linked = true;
          break;
        }
        if (linked)
          break;
      }
    }
  ProgramGraph g;
  for (const auto &entry : edgeSet)
    g.edges.push_back({entry.first.first, entry.first.second});
  Reachability reach(n, g.edges);
  std::vector<NodeId> dispatches;
  for (NodeId id = 0; id < n; ++id)
    if (nodes[id].kind == NodeKind::Dispatch)
      dispatches.push_back(id);
  for (NodeId target : dispatches) {
    std::vector<NodeId> kept;
    for (NodeId candidate : dispatches) {
      if (candidate >= target || !reach(candidate, target))
        continue;
      bool transitive = false;
      for (NodeId mid : dispatches)
        if (candidate < mid && mid < target && reach(candidate, mid) && reach(mid, target)) {
          transitive = true;
          break;
        }
      if (!transitive)
        kept.push_back(candidate);
    }
    g.dependencies[target] = std::move(kept);
  }
  // Resources in first-access order over dispatch nodes, with their dispatch users.
  g.users.assign(resources.size(), {});
  std::vector<bool> seen(resources.size(), false);
  for (NodeId id : dispatches)
    for (const BoundAccess &a : nodes[id].accesses) {
      if (!seen[a.resource]) {
        seen[a.resource] = true;
        g.resourceOrder.push_back(a.resource);
      }
      auto &u = g.users[a.resource];
      if (u.empty() || u.back() != id)
        u.push_back(id);
    }
  std::vector<PlannerResource> planned;
  for (ResourceId r : g.resourceOrder) {
    if (!resources[r].temporary)
      continue;
    PlannerResource pr;
    pr.name = "r" + std::to_string(r);
    pr.bytes = resources[r].bytes;
    pr.alignment = resources[r].alignment;
    pr.device = resources[r].device;
    pr.kind = resources[r].persistent ? ResourceKind::Persistent : ResourceKind::Temporary;
    pr.users = g.users[r];
    planned.push_back(std::move(pr));
    g.plannerToProgram.push_back(r);
  }
  g.memory = MemoryPlanner(reuseStorage).plan(n, g.edges, planned);
  return g;
}

// ---------------------------------------------------------------------------------------
// Repetition of a dependency list: iteration k+1's roots depend on all of iteration k's
// leaves (lib/Core/ExecutionPlan.cpp:87-117).
inline std::vector<std::vector<NodeId>> repeatDependencies(
    const std::vector<std::vector<NodeId>> &deps, std::size_t iterations) {
  if (!iterations)
    throw std::invalid_argument("execution plan repeat count must be nonzero");
  if (deps.empty())
    throw std::invalid_argument("cannot repeat an empty execution plan");
  const std::size_t n = deps.size();
  std::vector<bool> hasSuccessor(n, false);
  for (const auto &d : deps)
    for (NodeId p : d) {
      if (p >= n)
        throw std::invalid_argument("kernel dependencies must reference earlier plan nodes");
      hasSuccessor[p] = true;
    }
  std::vector<NodeId> leaves;
  for (NodeId i = 0; i < n; ++i)
    if (!hasSuccessor[i])
      leaves.push_back(i);
  std::vector<std::vector<NodeId>> out;
  out.reserve(n * iterations);
  for (std::size_t it = 0; it < iterations; ++it) {
    const std::size_t base = it * n;
    for (NodeId i = 0; i < n; ++i) {
      std::vector<NodeId> d;
      for (NodeId p : deps[i])
        d.push_back(base + p);
      if (it && deps[i].empty())
        for (NodeId leaf : leaves)
          d.push_back(base - n + leaf);
      out.push_back(std::move(d));
    }
  }
  return out;
}

} // namespace ckl::planning
