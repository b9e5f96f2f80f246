// Host-side geometry for the DTEM spatial routing library.
//
// The padded neighbour table restates build_patch_spatial_adjacency +
// adjacency_to_padded_neighbors (opentome/timm/dtem.py:50-127): row-major
// patches, squared grid distance compared in float32 with radius*radius,
// neighbours listed in ascending patch order, padding index 0 / invalid.
//
// The routing tables specialise that table to the canonical eval grouping
// (alternating_per_layer_fast, dtem.py:1170-1174 and :1811-1843): at layer
// parity q the donors are the patches of parity dp = (q ? 0 : 1) and the
// receivers the patches of the other parity, each group in ascending order.
// A donor's legal receivers are its static neighbours of receiver parity (the
// sorted-receiver binary search of dtem.py:399-422 finds exactly those).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/mergenet_b200.h"

namespace {

bool valid_grid(int h, int w, double radius) {
  return h > 0 && w > 0 && (long long)h * w <= (1 << 24) && std::isfinite(radius) && radius > 0.0;
}

// Neighbour lists of every patch, ascending.
void neighbor_lists(int h, int w, double radius, std::vector<std::vector<int>>& out) {
  const int P = h * w;
  const float r2 = (float)(radius * radius);
  // one row/column beyond floor(radius): the float32 comparison decides
  const int reach = (int)std::floor(radius) + 1;
  out.assign(P, {});
  for (int p = 0; p < P; ++p) {
    const int pr = p / w, pc = p % w;
    for (int rr = std::max(0, pr - reach); rr <= std::min(h - 1, pr + reach); ++rr) {
      for (int cc = std::max(0, pc - reach); cc <= std::min(w - 1, pc + reach); ++cc) {
        const long long dr = pr - rr, dc = pc - cc;
        if ((float)(dr * dr + dc * dc) <= r2) out[p].push_back(rr * w + cc);
      }
    }
  }
}

struct Parity {
  std::vector<std::vector<int>> slot_k, slot_rx;  // per donor: compact slots
  std::vector<std::vector<int>> rx_in;             // per receiver: edge ids
  std::vector<std::vector<int>> rx_off;            // per receiver: stencil offset index
};

// Stencil offsets of a receiver's donors for an even-width grid: donor
// columns differ by an odd dx.  Order: dx ascending over odd values, then dy
// ascending.  Returns -1 when (dy, dx) is outside the stencil.
int stencil_index(int dy, int dx, int dy1, int dy3) {
  int idx = 0;
  const int dxs[4] = {-3, -1, 1, 3};
  for (int i = 0; i < 4; ++i) {
    const int lim = (dxs[i] == -3 || dxs[i] == 3) ? dy3 : dy1;
    if (lim < 0) continue;
    for (int y = -lim; y <= lim; ++y) {
      if (dxs[i] == dx && y == dy) return idx;
      ++idx;
    }
  }
  return -1;
}

void build_parity(int h, int w, double radius, int q, const std::vector<std::vector<int>>& nbr,
                  int kc_stride, Parity& out, int* kc_max, int* kin_max, int* valid_rows) {
  const int P = h * w, half = P / 2;
  const int dp = q ? 0 : 1, rp = 1 - dp;
  out.slot_k.assign(half, {});
  out.slot_rx.assign(half, {});
  out.rx_in.assign(half, {});
  out.rx_off.assign(half, {});
  int kc = 0, rows = 0;
  for (int d = 0; d < half; ++d) {
    const int pd = 2 * d + dp;
    const auto& lst = nbr[pd];
    for (int k = 0; k < (int)lst.size(); ++k) {
      const int n = lst[k];
      if ((n & 1) == rp) {
        out.slot_k[d].push_back(k);
        out.slot_rx[d].push_back(n >> 1);
      }
    }
    kc = std::max(kc, (int)out.slot_k[d].size());
    rows += out.slot_k[d].empty() ? 0 : 1;
  }
  const int stride = kc_stride > 0 ? kc_stride : kc;
  for (int d = 0; d < half; ++d)
    for (int c = 0; c < (int)out.slot_rx[d].size(); ++c) {
      const int s = out.slot_rx[d][c];
      out.rx_in[s].push_back(d * stride + c);
      const int pd = 2 * d + dp, ps = 2 * s + rp;
      out.rx_off[s].push_back(pd / w - ps / w);      // dy, resolved to an index below
      out.rx_off[s].push_back(pd % w - ps % w);      // dx
    }
  int kin = 0;
  for (int s = 0; s < half; ++s) kin = std::max(kin, (int)out.rx_in[s].size());
  *kc_max = kc;
  *kin_max = kin;
  *valid_rows = rows;
  (void)radius;
}

}  // namespace

extern "C" int mn_version(void) { return 1; }

extern "C" int mn_neighbor_table_width(int grid_h, int grid_w, double radius, int* k_out) {
  if (!k_out || !valid_grid(grid_h, grid_w, radius)) return MN_ERR_ARG;
  std::vector<std::vector<int>> nbr;
  neighbor_lists(grid_h, grid_w, radius, nbr);
  int k = 0;
  for (const auto& l : nbr) k = std::max(k, (int)l.size());
  *k_out = k;
  return MN_OK;
}

extern "C" int mn_neighbor_table_fill(int grid_h, int grid_w, double radius, int k, int64_t* indices,
                                      uint8_t* valid) {
  if (!indices || !valid || !valid_grid(grid_h, grid_w, radius) || k <= 0) return MN_ERR_ARG;
  std::vector<std::vector<int>> nbr;
  neighbor_lists(grid_h, grid_w, radius, nbr);
  const int P = grid_h * grid_w;
  for (int p = 0; p < P; ++p) {
    if ((int)nbr[p].size() > k) return MN_ERR_ARG;
    for (int j = 0; j < k; ++j) {
      const bool v = j < (int)nbr[p].size();
      indices[(int64_t)p * k + j] = v ? nbr[p][j] : 0;
      valid[(int64_t)p * k + j] = v ? 1 : 0;
    }
  }
  return MN_OK;
}

extern "C" int mn_route_dims_query(int grid_h, int grid_w, double radius, mn_route_dims* dims) {
  if (!dims || !valid_grid(grid_h, grid_w, radius)) return MN_ERR_ARG;
  const int P = grid_h * grid_w;
  if (P % 2 != 0 || P < 2) return MN_ERR_UNSUPPORTED;
  std::vector<std::vector<int>> nbr;
  neighbor_lists(grid_h, grid_w, radius, nbr);
  std::memset(dims, 0, sizeof(*dims));
  dims->grid_h = grid_h;
  dims->grid_w = grid_w;
  dims->num_patches = P;
  dims->half = P / 2;
  for (const auto& l : nbr) dims->k_static = std::max(dims->k_static, (int)l.size());
  for (int p = 0; p < P; ++p)
    for (int n : nbr[p]) dims->radius_rows = std::max(dims->radius_rows, std::abs(n / grid_w - p / grid_w));
  int kc = 0, kin = 0;
  for (int q = 0; q < 2; ++q) {
    Parity par;
    int a, b, rows;
    build_parity(grid_h, grid_w, radius, q, nbr, 0, par, &a, &b, &rows);
    kc = std::max(kc, a);
    kin = std::max(kin, b);
    dims->valid_rows[q] = rows;
  }
  dims->kc = std::max(kc, 1);
  dims->kin = std::max(kin, 1);
  // Stencil form of the feature transport: even width (patch parity =
  // column parity), donors at odd dx in {-3,-1,1,3}; dy limits per |dx|.
  int dy1 = -1, dy3 = -1;
  bool ok = (grid_w % 2) == 0;
  for (int q = 0; q < 2 && ok; ++q) {
    Parity par;
    int a, b, rows;
    build_parity(grid_h, grid_w, radius, q, nbr, 0, par, &a, &b, &rows);
    for (int s = 0; s < dims->half && ok; ++s)
      for (size_t j = 0; j + 1 < par.rx_off[s].size(); j += 2) {
        const int dy = std::abs(par.rx_off[s][j]), dx = std::abs(par.rx_off[s][j + 1]);
        if (dx == 1) dy1 = std::max(dy1, dy);
        else if (dx == 3) dy3 = std::max(dy3, dy);
        else ok = false;
      }
  }
  dims->stencil_dy1 = ok ? dy1 : -2;
  dims->stencil_dy3 = ok ? dy3 : -2;
  dims->table_ints = (int64_t)2 * ((int64_t)dims->half * dims->kc * 2 + (int64_t)dims->half * dims->kin * 2);
  return MN_OK;
}

extern "C" int mn_route_tables_fill(int grid_h, int grid_w, double radius, const mn_route_dims* dims,
                                    int32_t* host_table) {
  if (!dims || !host_table) return MN_ERR_ARG;
  mn_route_dims check;
  int rc = mn_route_dims_query(grid_h, grid_w, radius, &check);
  if (rc != MN_OK) return rc;
  if (check.half != dims->half || check.kc != dims->kc || check.kin != dims->kin) return MN_ERR_ARG;
  std::vector<std::vector<int>> nbr;
  neighbor_lists(grid_h, grid_w, radius, nbr);
  const int half = dims->half, kc = dims->kc, kin = dims->kin;
  int32_t* t = host_table;
  for (int q = 0; q < 2; ++q) {
    Parity par;
    int a, b, rows;
    build_parity(grid_h, grid_w, radius, q, nbr, kc, par, &a, &b, &rows);
    int32_t* sk = t;
    int32_t* sr = t + (int64_t)half * kc;
    int32_t* ri = t + (int64_t)half * kc * 2;
    int32_t* ro = ri + (int64_t)half * kin;
    for (int d = 0; d < half; ++d)
      for (int c = 0; c < kc; ++c) {
        const bool v = c < (int)par.slot_k[d].size();
        sk[(int64_t)d * kc + c] = v ? par.slot_k[d][c] : -1;
        sr[(int64_t)d * kc + c] = v ? par.slot_rx[d][c] : -1;
      }
    for (int s = 0; s < half; ++s)
      for (int j = 0; j < kin; ++j) {
        const bool v = j < (int)par.rx_in[s].size();
        ri[(int64_t)s * kin + j] = v ? par.rx_in[s][j] : -1;
        ro[(int64_t)s * kin + j] =
            (v && dims->stencil_dy1 >= -1)
                ? stencil_index(par.rx_off[s][2 * j], par.rx_off[s][2 * j + 1], dims->stencil_dy1, dims->stencil_dy3)
                : -1;
      }
    t += (int64_t)half * kc * 2 + (int64_t)half * kin * 2;
  }
  return MN_OK;
}
