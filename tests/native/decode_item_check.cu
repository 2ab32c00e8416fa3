// CPU check of the persistent kernels' work-item decode (tiledattention_b200/csrc/
// sdpa_common.cuh, decode_item): compiled with nvcc and run on the host by
// tests/test_decode_item_cpu.py. For every configuration in a sweep it checks that
//   - every (key slice, (b,h) pair, query block) is decoded exactly once;
//   - items come slice by slice, then group by group of group_bh pairs, and inside a group
//     the query blocks never get later (longest causal blocks first);
//   - b, h, q_row0, the key range and the key-tile count are what the mask and the slice
//     bounds imply.
// Prints "ok <configurations>" or the first violation, and exits non-zero on one.
#include <cstdio>
#include <vector>

#include "../../tiledattention_b200/csrc/sdpa_common.cuh"

using ta::FwdParams;
using ta::common::Item;

template <bool CAUSAL, int kRows>
static bool check(int B, int H, int S, int group_bh, int kv_begin, int kv_end, int n_split) {
  constexpr int kKeys = 128;
  FwdParams p{};
  p.S = S;
  p.H = H;
  p.BH = B * H;
  p.n_qblk = (S + kRows - 1) / kRows;
  p.kv_begin = kv_begin;
  p.kv_end = kv_end;
  p.n_split = n_split;
  const int span = kv_end - kv_begin;
  int split_len = (span + n_split - 1) / n_split;
  split_len = (split_len + kKeys - 1) / kKeys * kKeys;
  p.split_len = split_len > 0 ? split_len : kKeys;
  p.group_bh = group_bh;
  const int n_items = n_split * p.BH * p.n_qblk;
  std::vector<int> seen(static_cast<size_t>(n_items), 0);
  int prev_split = -1, prev_group = -1, prev_qrow = 0;
  for (int item = 0; item < n_items; ++item) {
    const Item it = ta::common::decode_item<CAUSAL, kRows, kKeys>(p, item);
    const int qblk = it.q_row0 / kRows;
    const bool in_range = it.split >= 0 && it.split < n_split && it.bh >= 0 && it.bh < p.BH &&
                          qblk >= 0 && qblk < p.n_qblk && it.q_row0 % kRows == 0;
    if (!in_range || it.b != it.bh / H || it.h != it.bh % H) {
      std::printf("FAIL out of range: item %d (split %d bh %d q_row0 %d)\n", item, it.split,
                  it.bh, it.q_row0);
      return false;
    }
    int& count = seen[(static_cast<size_t>(it.split) * p.BH + it.bh) * p.n_qblk + qblk];
    if (++count != 1) {
      std::printf("FAIL item %d decodes a unit twice\n", item);
      return false;
    }
    const int group = it.bh / group_bh;
    if (it.split < prev_split || (it.split == prev_split && group < prev_group)) {
      std::printf("FAIL item %d: slice/group order\n", item);
      return false;
    }
    if (it.split == prev_split && group == prev_group && it.q_row0 > prev_qrow) {
      std::printf("FAIL item %d: a later query block after an earlier one in a group\n", item);
      return false;
    }
    prev_split = it.split;
    prev_group = group;
    prev_qrow = it.q_row0;
    const int lo = kv_begin + it.split * p.split_len < kv_end ? kv_begin + it.split * p.split_len
                                                              : kv_end;
    const int hi = lo + p.split_len < kv_end ? lo + p.split_len : kv_end;
    const int rows = CAUSAL ? (hi < it.q_row0 + kRows ? hi : it.q_row0 + kRows) : hi;
    const int n_kv = rows > lo ? (rows - lo + kKeys - 1) / kKeys : 0;
    if (it.kv_lo != lo || it.kv_hi != hi || it.n_kv != n_kv || it.kv_lo < kv_begin ||
        it.kv_hi > kv_end) {
      std::printf("FAIL item %d: key range [%d,%d) n_kv %d, expected [%d,%d) %d\n", item,
                  it.kv_lo, it.kv_hi, it.n_kv, lo, hi, n_kv);
      return false;
    }
  }
  return true;
}

int main() {
  int configs = 0;
  const int shapes[][3] = {{1, 1, 1}, {1, 2, 64}, {2, 3, 1000}, {1, 8, 4096}, {8, 32, 4096},
                           {2, 4, 3001}, {1, 16, 65536}, {3, 5, 129}};
  for (const auto& sh : shapes) {
    const int B = sh[0], H = sh[1], S = sh[2];
    const int BH = B * H;
    const int groups[] = {1, 2, 3, 7, 16, BH};
    for (int g : groups) {
      if (g > BH) continue;
      const int splits[] = {1, 2, 3, 4};
      for (int n : splits) {
        const int ranges[][2] = {{0, S}, {S / 3, S}, {0, (S + 1) / 2}};
        for (const auto& r : ranges) {
          if (r[1] <= r[0]) continue;
          bool ok = check<true, 128>(B, H, S, g, r[0], r[1], n) &&
                    check<false, 128>(B, H, S, g, r[0], r[1], n) &&
                    check<true, 256>(B, H, S, g, r[0], r[1], n) &&
                    check<false, 256>(B, H, S, g, r[0], r[1], n);
          if (!ok) {
            std::printf("config B=%d H=%d S=%d group_bh=%d kv=[%d,%d) n_split=%d\n", B, H, S, g,
                        r[0], r[1], n);
            return 1;
          }
          configs += 4;
        }
      }
    }
  }
  std::printf("ok %d\n", configs);
  return 0;
}
