// level_plan.cpp -- C-ABI check and launch shape of a lowered level-graph plan.
#include <cstring>

#include "common.hpp"

using namespace to_b200;

extern "C" int to_level_plan_lower(const to_level_plan_desc* d, int32_t query_device,
                                   to_level_launch* out) {
  if (!d || !out) return set_error(TO_ERR_INVALID_ARGUMENT, "to_level_plan_lower: null");
  std::memset(out, 0, sizeof(*out));
  if (d->value_bytes <= 0 || d->num_levels < 0 || d->num_slots < 0 || d->num_pools < 0 ||
      d->grid_rank < 0 || d->num_whole < 0)
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_level_plan_lower: negative count");
  if ((d->num_levels && (!d->level_kind || !d->level_members || !d->level_space)) ||
      (d->num_slots && (!d->slot_def || !d->slot_last || !d->slot_pool || !d->slot_bytes)) ||
      !d->pool_offset || (d->grid_rank && (!d->grid_extent || !d->grid_tile)) ||
      (d->num_whole && (!d->whole_extent || !d->whole_tile)))
    return set_error(TO_ERR_INVALID_ARGUMENT, "to_level_plan_lower: null table");
  if (d->grid_rank == 0)
    return set_error(TO_ERR_INVALID_ARGUMENT,
                     "level graph: at least one label must be blocked (LabelTile) -- with every "
                     "label declared LabelWhole the whole problem is one team");
  // levels
  int64_t widest = 1;
  for (int l = 0; l < d->num_levels; ++l) {
    if (d->level_kind[l] < 0 || d->level_kind[l] > 3 || d->level_members[l] <= 0)
      return set_error(TO_ERR_INVALID_ARGUMENT, "level %d: bad kind or empty", l);
    if (d->level_space[l] <= 0)
      return set_error(TO_ERR_INVALID_ARGUMENT, "level %d: empty iteration space", l);
    if (d->level_space[l] > widest) widest = d->level_space[l];
  }
  // pools: offsets increasing, every slot fits its pool, live ranges in a pool disjoint
  for (int q = 0; q < d->num_pools; ++q)
    if (d->pool_offset[q + 1] < d->pool_offset[q] || d->pool_offset[q] % 16)
      return set_error(TO_ERR_INVALID_ARGUMENT, "pool %d: offset not increasing / 16-aligned", q);
  for (int s = 0; s < d->num_slots; ++s) {
    const int q = d->slot_pool[s];
    if (q < 0 || q >= d->num_pools)
      return set_error(TO_ERR_INVALID_ARGUMENT, "slot %d: pool %d out of range", s, q);
    if (d->slot_def[s] < 0 || d->slot_def[s] >= d->num_levels || d->slot_last[s] < d->slot_def[s] ||
        d->slot_last[s] > d->num_levels)
      return set_error(TO_ERR_INVALID_ARGUMENT, "slot %d: live range [%d, %d] invalid", s,
                       d->slot_def[s], d->slot_last[s]);
    if (d->slot_bytes[s] > d->pool_offset[q + 1] - d->pool_offset[q])
      return set_error(TO_ERR_INVALID_ARGUMENT, "slot %d: %lld bytes do not fit pool %d", s,
                       static_cast<long long>(d->slot_bytes[s]), q);
    for (int t = 0; t < s; ++t)
      if (d->slot_pool[t] == q && !(d->slot_last[t] < d->slot_def[s] ||
                                    d->slot_last[s] < d->slot_def[t]))
        return set_error(TO_ERR_INVALID_ARGUMENT,
                         "slots %d and %d share pool %d but are live together (levels [%d,%d] "
                         "and [%d,%d])",
                         t, s, q, d->slot_def[t], d->slot_last[t], d->slot_def[s], d->slot_last[s]);
  }
  // grid
  int64_t league = 1;
  for (int g = 0; g < d->grid_rank; ++g) {
    if (d->grid_tile[g] <= 0 || d->grid_extent[g] < 0)
      return set_error(TO_ERR_INVALID_ARGUMENT, "grid label %d: bad extent/tile", g);
    league *= (d->grid_extent[g] + d->grid_tile[g] - 1) / d->grid_tile[g];
  }
  for (int w = 0; w < d->num_whole; ++w)
    if (d->whole_extent[w] > d->whole_tile[w])
      return set_error(TO_ERR_GRID,
                       "level graph: a label declared LabelWhole is longer than its tile "
                       "(%lld > %d), so it needs to be gridded -- declare it LabelTile instead",
                       static_cast<long long>(d->whole_extent[w]), d->whole_tile[w]);
  if (league > 2147483647ll)
    return set_error(TO_ERR_INVALID_ARGUMENT, "league of %lld teams exceeds the grid limit",
                     static_cast<long long>(league));
  int team = d->team_size;
  if (team > 1024) return set_error(TO_ERR_INVALID_ARGUMENT, "team size %d > 1024", team);
  if (team <= 0) {
    const int64_t r = ((widest + 31) / 32) * 32;
    team = static_cast<int>(r < 64 ? 64 : (r > 512 ? 512 : r));
  }
  const int64_t scratch = d->num_pools ? d->pool_offset[d->num_pools] : 0;
  if (query_device) {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    if (scratch > optin)
      return set_error(TO_ERR_SCRATCH,
                       "level graph needs %lld B of team scratch per CTA, the device allows %d",
                       static_cast<long long>(scratch), optin);
  }
  out->league = league;
  out->team = team;
  out->scratch_bytes = scratch;
  return ok();
}
