// kq_ngram.h -- prompt-lookup drafter (host side): proposes the tokens that followed the latest
// earlier occurrence of the longest matching suffix of the token history, suffix lengths
// nmax .. nmin. Behaviour of the reference's NgramDraft (scripts/kindi_q4/kindi/spec.py:801-841):
//  - push(t) appends t and indexes every n-gram (nmin <= n <= nmax) that ends just before t by
//    the position of t, so each indexed n-gram points at an existing continuation, the latest
//    one winning;
//  - truncate(L) drops positions >= L; index entries that point past the end or at a changed
//    n-gram are recognised when looked up, not removed;
//  - propose(k), for n = nmax down to nmin: skip a suffix that holds a -1 (an unknown token);
//    take the indexed position j of the suffix if j is inside the history, j >= n and the n
//    tokens before j still equal the suffix; the proposal is then the up to k tokens from j on,
//    empty if one of them is -1, other negative tokens left out. No match at any n: empty.
// The index is a hash map keyed by the n-gram's bytes (n-grams of different lengths never
// collide: their keys differ in length).
#pragma once
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace kq {

class NgramIndex {
 public:
  NgramIndex(int nmax, int nmin) : nmax_(nmax), nmin_(nmin) {}

  void reset(const int32_t* hist, int n) {
    idx_.clear();
    h_.clear();
    for (int i = 0; i < n; ++i) push(hist[i]);
  }
  void truncate(int L) {
    if (L < (int)h_.size()) h_.resize((size_t)L);
  }
  void push(int32_t t) {
    h_.push_back(t);
    const int L = (int)h_.size();
    for (int n = nmin_; n <= nmax_; ++n)
      if (L - 1 - n >= 0) idx_[key(L - 1 - n, n)] = L - 1;
  }
  // Writes the proposal to out (at most k tokens) and returns its length.
  int propose(int k, int32_t* out) const {
    const int L = (int)h_.size();
    for (int n = nmax_; n >= nmin_; --n) {
      if (L < n) continue;
      bool unknown = false;
      for (int i = L - n; i < L; ++i) unknown |= h_[i] == -1;
      if (unknown) continue;
      const auto it = idx_.find(key(L - n, n));
      if (it == idx_.end()) continue;
      const int j = it->second;
      if (j >= L || j < n || std::memcmp(&h_[j - n], &h_[L - n], (size_t)n * sizeof(int32_t)) != 0) continue;
      const int e = j + k < L ? j + k : L;
      for (int i = j; i < e; ++i)
        if (h_[i] == -1) return 0;
      int m = 0;
      for (int i = j; i < e; ++i)
        if (h_[i] >= 0) out[m++] = h_[i];
      return m;
    }
    return 0;
  }
  int length() const { return (int)h_.size(); }

 private:
  std::string key(int start, int n) const {
    return std::string(reinterpret_cast<const char*>(&h_[(size_t)start]), (size_t)n * sizeof(int32_t));
  }
  int nmax_, nmin_;
  std::vector<int32_t> h_;
  std::unordered_map<std::string, int> idx_;
};

}  // namespace kq
