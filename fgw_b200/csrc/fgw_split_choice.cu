// Host-side split choice of the B200 (version-3) split cost model, for callers that hand the library the
// host copy of their cache lengths every call (a serving loop): one pass over the lengths gives their range
// check, whether every cache is full, and the 128-token KV-tile sum and maximum the model reads; the model's
// predicted latency per candidate split count then picks the smallest count within the selection tolerance of
// the best. This is the choice FGW makes in Python on the host before every launch
// (operators/mha/general_split_cost_model.py:70-91, `predict_us` / `select_model_splits`), with the B200
// model's features; the Python restatement (fgw_b200/operators/mha/general_split_cost_model.py,
// `select_b200_splits`) makes the same choice, and a CPU test holds the two to identical picks.
//
// The arithmetic follows the Python order of operations in double precision, so predictions (and ties) are
// the same bits: features are accumulated left to right into the sum of weight x feature products.
#include <algorithm>
#include <cmath>
#include <cstdint>

#include "fgw_kernels.h"

namespace fgw {
namespace {

constexpr int kCandidates[] = {1, 2, 4, 8, 16, 32, 64, 128};  // B200_SPLITS
constexpr int kDecodeMaxQueries = 8;
constexpr int kPairRows = 256;
constexpr int kKvTile = 128;

// The model's ten features (FEATURE_NAMES_V3) for one candidate split count.
void features(int batch, int sq, int heads, int dim, long long tiles_sum, long long tiles_max, int splits, int cores,
              double (&f)[FGW_SPLIT_MODEL_FEATURES]) {
  const double mean_tiles = static_cast<double>(tiles_sum) / static_cast<double>(batch);
  const bool decode = sq <= kDecodeMaxQueries;
  const int rows = decode ? decode_rows_per_item(dim) : kPairRows;
  const long long items = static_cast<long long>(batch) * heads * ((sq + rows - 1) / rows) * splits;
  double pieces = 0.0;
  double serial, waves;
  if (!decode && splits == 1 && 3 * items < 2ll * kStreamMaxPrograms) {
    const int programs = std::min(cores, kStreamMaxPrograms);
    serial = std::ceil(static_cast<double>(items) * std::max(mean_tiles, 1.0) / static_cast<double>(programs));
    waves = 1.0;
    pieces = std::min(static_cast<double>(programs) / static_cast<double>(items), std::max(mean_tiles, 1.0));
  } else {
    const long long w = (items + cores - 1) / cores;
    waves = static_cast<double>(w);
    serial = static_cast<double>(w * static_cast<long long>(std::ceil(mean_tiles / static_cast<double>(splits))));
  }
  const long long longest = (tiles_max + splits - 1) / splits;
  const int multi = splits > 1 ? 1 : 0;
  f[0] = 1.0;
  f[1] = decode ? serial : 0.0;
  f[2] = decode ? 0.0 : serial;
  f[3] = decode ? waves : 0.0;
  f[4] = decode ? 0.0 : waves;
  f[5] = static_cast<double>(multi);
  f[6] = static_cast<double>(splits);
  f[7] = static_cast<double>(static_cast<long long>(multi) * batch * heads * sq * splits) / static_cast<double>(cores);
  f[8] = std::max(0.0, static_cast<double>(longest) - mean_tiles / static_cast<double>(splits));
  f[9] = pieces;
}

}  // namespace
}  // namespace fgw

using namespace fgw;

extern "C" int fgw_mha_choose_splits(const fgw_split_model* model, const int32_t* host_lengths, int batch, int q_len,
                                     int heads, int head_dim, int page_size, int table_width, int sm_count,
                                     fgw_split_choice* choice) {
  if (model == nullptr || choice == nullptr || (host_lengths == nullptr && batch > 0)) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  if (batch <= 0 || q_len <= 0 || heads <= 0 || head_dim <= 0 || page_size <= 0 || table_width <= 0 ||
      sm_count <= 0) {
    return FGW_ERR_INVALID_ARGUMENT;
  }
  const long long capacity = static_cast<long long>(page_size) * table_width;
  long long tiles_sum = 0, tiles_max = 0;
  int32_t lo = host_lengths[0], hi = host_lengths[0];
  for (int b = 0; b < batch; ++b) {
    const int32_t n = host_lengths[b];
    lo = std::min(lo, n);
    hi = std::max(hi, n);
    const long long tiles = (static_cast<long long>(n) + kKvTile - 1) / kKvTile;
    tiles_sum += tiles;
    tiles_max = std::max(tiles_max, tiles);
  }
  choice->min_length = lo;
  choice->max_length = hi;
  choice->full_kv_cache = lo == capacity ? 1 : 0;
  choice->splits = 0;
  if (lo < 0 || hi > capacity) return FGW_ERR_INVALID_ARGUMENT;  // "Cache lengths must be within table capacity"
  const long long capacity_tiles = (capacity + kKvTile - 1) / kKvTile;
  double best = INFINITY;
  double cost[sizeof(kCandidates) / sizeof(kCandidates[0])];
  int count = 0;
  for (int s : kCandidates) {
    if (s > capacity_tiles) break;
    double f[FGW_SPLIT_MODEL_FEATURES];
    features(batch, q_len, heads, head_dim, tiles_sum, tiles_max, s, sm_count, f);
    double raw = 0.0;
    for (int i = 0; i < FGW_SPLIT_MODEL_FEATURES; ++i) raw += f[i] * model->weights[i];
    const double floor = s > 1 ? model->floor_multi_us : model->floor_single_us;
    cost[count] = std::max(raw, floor);
    best = std::min(best, cost[count]);
    ++count;
  }
  const double limit = best + std::max(best * model->tolerance, model->absolute_margin_us);
  for (int i = 0; i < count; ++i) {
    if (cost[i] <= limit) {
      choice->splits = kCandidates[i];
      break;
    }
  }
  return FGW_OK;
}
