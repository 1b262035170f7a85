// Connected components of equal positive labels, 6-connectivity (4 in 2-D), on the host.
//
// Runs inside dataloader worker processes so the training device never waits on a data-dependent
// number of rounds (the device alternative in the reference needs a host sync per round,
// src/algorithms/affinity/targets.py:40-108). Classic two-pass labelling with a union-find over
// provisional ids (path halving, union by smaller root): pass one scans in raster order and joins
// each voxel with its already-visited neighbours (-x, -y, -z) that carry the same positive id;
// pass two resolves roots and numbers components 1..K in order of first appearance.
// Background (0) and ignore (negative) voxels are copied through unchanged.
#include <torch/extension.h>

#include <cstdint>
#include <vector>

namespace mia {

namespace {

struct UnionFind {
  std::vector<int64_t> parent;
  int64_t make() {
    parent.push_back((int64_t)parent.size());
    return (int64_t)parent.size() - 1;
  }
  int64_t find(int64_t a) {
    while (parent[a] != a) {
      parent[a] = parent[parent[a]];
      a = parent[a];
    }
    return a;
  }
  void unite(int64_t a, int64_t b) {
    a = find(a);
    b = find(b);
    if (a == b) return;
    if (a < b) parent[b] = a; else parent[a] = b;
  }
};

template <typename L>
void label_components(const L* in, int64_t* out, int64_t X, int64_t Y, int64_t Z) {
  const int64_t n = X * Y * Z;
  std::vector<int64_t> prov(n, -1);
  UnionFind uf;
  uf.parent.reserve(1024);
  for (int64_t x = 0; x < X; ++x)
    for (int64_t y = 0; y < Y; ++y)
      for (int64_t z = 0; z < Z; ++z) {
        const int64_t i = (x * Y + y) * Z + z;
        const int64_t v = (int64_t)in[i];
        if (v <= 0) continue;
        int64_t id = -1;
        const int64_t nbrs[3] = {z > 0 ? i - 1 : -1, y > 0 ? i - Z : -1, x > 0 ? i - Y * Z : -1};
        for (int64_t j : nbrs) {
          if (j < 0 || (int64_t)in[j] != v) continue;
          if (id < 0) id = prov[j]; else uf.unite(id, prov[j]);
        }
        prov[i] = id >= 0 ? id : uf.make();
      }
  std::vector<int64_t> dense(uf.parent.size(), 0);
  int64_t next = 0;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t v = (int64_t)in[i];
    if (v <= 0) {
      out[i] = v;
      continue;
    }
    const int64_t r = uf.find(prov[i]);
    if (dense[r] == 0) dense[r] = ++next;
    out[i] = dense[r];
  }
}

}  // namespace

at::Tensor connected_components_cpu(at::Tensor labels) {
  TORCH_CHECK(labels.device().is_cpu(), "connected_components_cpu: a CPU tensor is expected");
  TORCH_CHECK(labels.dim() >= 1 && labels.dim() <= 3, "connected_components_cpu: 1-3 spatial axes expected");
  auto in = labels.contiguous();
  int64_t dims[3] = {1, 1, 1};
  for (int64_t d = 0; d < in.dim(); ++d) dims[3 - in.dim() + d] = in.size(d);
  auto out = at::empty(in.sizes(), in.options().dtype(at::kLong));
  AT_DISPATCH_INTEGRAL_TYPES(in.scalar_type(), "connected_components_cpu", [&] {
    label_components<scalar_t>(in.data_ptr<scalar_t>(), out.data_ptr<int64_t>(), dims[0], dims[1], dims[2]);
  });
  return out;
}

}  // namespace mia
