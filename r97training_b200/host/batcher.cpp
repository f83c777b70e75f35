// batcher.cpp -- the token-budget batcher of the training loop, as a C entry point of libr97host.so.
//
// The plan of an epoch must be the reference's exactly (include/r97/batcher.h, src/batcher.cpp): a run
// resumed from a saved (epoch, step) position, or a data-parallel job whose ranks each take sub-batch
// `rank` of every step, has to hand out the same sequences the reference would, so the grouping, the
// splitmix64 streams and their seeds, both shuffles, the packer's rules and the fixed-length step plan are
// restated here step for step. The batcher plans from the sequences' token counts alone and hands out
// indices; the caller (r97training_b200/data.py) holds the sequences.
//
//   1. Kept sequences (token count <= budget) sorted by count, longest first, ties by input index, then cut
//      into buckets of at most 32 that never straddle a power-of-two length class (bit width of the count).
//   2. More than one bucket: each bucket shuffled (Fisher-Yates) from a stream for (seed, epoch, bucket),
//      the bucket order shuffled from the (seed, epoch) stream and rotated to start on the bucket the seed's
//      hash plus the epoch names. One bucket: its first sequence is the one the seed's hash plus the epoch
//      names, the rest a Fisher-Yates under (seed, epoch).
//   3. Adjacent buckets of one class merge into a run. A single run of one positive length gets the exact
//      fixed-length plan; otherwise the runs are packed greedily: a sequence goes to the least-loaded
//      sub-batch (ties: lowest device) that is not sealed, holds its class or nothing, stays under the
//      budget and keeps the step's spread inside one maximal sequence -- an add landing exactly on that
//      bound is admitted only when the run's next sequences can raise the step's bottom. A run ending with
//      fewer sub-batches than devices carries into the next run with its occupied devices sealed.
#include <algorithm>
#include <bit>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace {

thread_local std::string g_batcher_error;

using Index = int64_t;
using SubBatch = std::vector<Index>;
using Step = std::vector<SubBatch>;
using Plan = std::vector<Step>;
using Run = std::vector<Index>;

// ------------------------------------------------------------------------------------------ streams
struct Mix64 {  // splitmix64
    uint64_t state;
    uint64_t next() {
        state += 0x9e3779b97f4a7c15ull;
        uint64_t z = state;
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        return z ^ (z >> 31);
    }
    uint64_t below(uint64_t n) { return next() % n; }
};

// The (seed, epoch) stream, warmed up by one draw.
Mix64 epoch_stream(uint64_t seed, int64_t epoch) {
    Mix64 m{seed ^ (0xd1b54a32d192ed03ull + (uint64_t)epoch * 0x9e3779b97f4a7c15ull)};
    m.next();
    return m;
}

// Which of n places the epoch starts on: the seed's hash, moved on by one an epoch.
size_t epoch_start(uint64_t seed, int64_t epoch, size_t n) {
    Mix64 m{seed ^ 0xa0761d6478bd642full};
    const uint64_t base = m.below((uint64_t)n);
    return (size_t)((base + (uint64_t)epoch % (uint64_t)n) % (uint64_t)n);
}

int length_class(int64_t tokens) { return (int)std::bit_width((uint64_t)tokens); }

// Fisher-Yates over v[lo, v.size()) with draws j = lo + below(i - lo + 1), i from the top down to lo + 1.
template <class T>
void shuffle_tail(std::vector<T>& v, size_t lo, Mix64& m) {
    for (size_t i = v.size(); i > lo + 1; --i) {
        const size_t j = lo + (size_t)m.below((uint64_t)(i - lo));
        std::swap(v[i - 1], v[j]);
    }
}

// ------------------------------------------------------------------------------------------ grouping
std::vector<Run> shuffled_buckets(std::vector<Index> order, const std::vector<int64_t>& lens, uint64_t seed,
                                  int64_t epoch) {
    std::sort(order.begin(), order.end(), [&](Index a, Index b) {
        return lens[a] != lens[b] ? lens[a] > lens[b] : a < b;
    });
    std::vector<Run> buckets;
    for (size_t lo = 0; lo < order.size();) {
        const int cls = length_class(lens[order[lo]]);
        size_t hi = lo + 1;
        while (hi < order.size() && hi - lo < 32 && length_class(lens[order[hi]]) == cls) ++hi;
        buckets.emplace_back(order.begin() + (std::ptrdiff_t)lo, order.begin() + (std::ptrdiff_t)hi);
        lo = hi;
    }
    const size_t nb = buckets.size();
    if (nb > 1) {
        for (size_t b = 0; b < nb; ++b) {
            Mix64 m = epoch_stream(seed ^ (0x2545f4914f6cdd1dull * (uint64_t)(b + 1)), epoch);
            shuffle_tail(buckets[b], 0, m);
        }
        std::vector<size_t> slot(nb);
        for (size_t i = 0; i < nb; ++i) slot[i] = i;
        Mix64 m = epoch_stream(seed, epoch);
        shuffle_tail(slot, 0, m);
        const size_t lead = epoch_start(seed, epoch, nb);
        const size_t at = (size_t)(std::find(slot.begin(), slot.end(), lead) - slot.begin());
        std::vector<Run> out;
        out.reserve(nb);
        for (size_t i = 0; i < nb; ++i) out.push_back(std::move(buckets[slot[(at + i) % nb]]));
        return out;
    }
    if (nb == 1 && buckets[0].size() > 1) {
        Run& only = buckets[0];
        std::swap(only[0], only[epoch_start(seed, epoch, only.size())]);
        Mix64 m = epoch_stream(seed, epoch);
        shuffle_tail(only, 1, m);
    }
    return buckets;
}

// ------------------------------------------------------------------------------------------ packing
class Packer {
public:
    Packer(const std::vector<int64_t>& lens, int64_t budget, int devices)
        : lens_(lens), budget_(budget), nd_((size_t)devices), subs_(nd_), load_(nd_, 0), sealed_(nd_, 0),
          cls_(nd_, -1) {}

    void pack_run(const Run& run, bool more_runs) {
        for (size_t i = 0; i < run.size(); ++i) {
            const Index s = run[i];
            const int cls = length_class(lens_[s]);
            size_t d = choose(s, cls, run, i + 1);
            if (d == kNone) {
                close();
                d = choose(s, cls, run, i + 1);
            }
            subs_[d].push_back(s);
            load_[d] += lens_[s];
            cls_[d] = cls;
            step_max_ = std::max(step_max_, lens_[s]);
        }
        const size_t used = occupied();
        if (used == 0) return;
        if (more_runs && used < nd_) {
            for (size_t k = 0; k < nd_; ++k) sealed_[k] = !subs_[k].empty();
        } else {
            close();
        }
    }

    Plan take() { return std::move(plan_); }

private:
    static constexpr size_t kNone = (size_t)-1;

    size_t occupied() const {
        size_t n = 0;
        for (const auto& s : subs_) n += !s.empty();
        return n;
    }

    void close() {
        Step step;
        for (auto& s : subs_)
            if (!s.empty()) step.push_back(std::move(s));
        if (!step.empty()) plan_.push_back(std::move(step));
        for (size_t k = 0; k < nd_; ++k) {
            subs_[k].clear();
            load_[k] = 0;
            sealed_[k] = 0;
            cls_[k] = -1;
        }
        step_max_ = 0;
    }

    // The least-loaded sub-batch that may take sequence s (the run's next unpacked one is run[next]).
    size_t choose(Index s, int cls, const Run& run, size_t next) const {
        size_t best = kNone;
        for (size_t k = 0; k < nd_; ++k) {
            if (sealed_[k] || (!subs_[k].empty() && cls_[k] != cls) || load_[k] + lens_[s] > budget_) continue;
            if (!spread_ok(s, k, cls, run, next)) continue;
            if (best == kNone || load_[k] < load_[best]) best = k;
        }
        return best;
    }

    // After s joins sub-batch d: the spread of the occupied sub-batches against the longest sequence.
    bool spread_ok(Index s, size_t d, int cls, const Run& run, size_t next) const {
        int64_t hi = load_[d] + lens_[s], lo = hi;
        size_t n = 1;
        for (size_t k = 0; k < nd_; ++k) {
            if (k == d || subs_[k].empty()) continue;
            hi = std::max(hi, load_[k]);
            lo = std::min(lo, load_[k]);
            ++n;
        }
        const int64_t longest = std::max(step_max_, lens_[s]);
        if (n < 2 || longest == 0 || hi - lo < longest) return true;
        if (hi - lo > longest) return false;
        for (size_t k = 0; k < nd_; ++k)
            if (!subs_[k].empty() && cls_[k] != cls) return false;  // a sealed bottom cannot be raised
        return bottom_rises(s, d, run, next);
    }

    // On the bound: whether the run's next sequences (at most one a device), each going to the least-loaded
    // sub-batch with room, bring the spread strictly inside it.
    bool bottom_rises(Index s, size_t d, const Run& run, size_t next) const {
        std::vector<int64_t> load = load_;
        std::vector<char> used(nd_);
        for (size_t k = 0; k < nd_; ++k) used[k] = !subs_[k].empty();
        load[d] += lens_[s];
        used[d] = 1;
        int64_t longest = std::max(step_max_, lens_[s]);
        for (size_t added = 0;; ++added) {
            int64_t hi = 0, lo = 0;
            size_t n = 0;
            for (size_t k = 0; k < nd_; ++k) {
                if (!used[k]) continue;
                hi = n ? std::max(hi, load[k]) : load[k];
                lo = n ? std::min(lo, load[k]) : load[k];
                ++n;
            }
            if (n < 2 || hi - lo < longest) return true;
            if (hi - lo > longest || added == nd_ || next + added >= run.size()) return false;
            const int64_t l = lens_[run[next + added]];
            size_t best = kNone;
            for (size_t k = 0; k < nd_; ++k)
                if (load[k] + l <= budget_ && (best == kNone || load[k] < load[best])) best = k;
            if (best == kNone) return false;
            load[best] += l;
            used[best] = 1;
            longest = std::max(longest, l);
        }
    }

    const std::vector<int64_t>& lens_;
    const int64_t budget_;
    const size_t nd_;
    std::vector<SubBatch> subs_;
    std::vector<int64_t> load_;
    std::vector<char> sealed_;
    std::vector<int> cls_;
    int64_t step_max_ = 0;
    Plan plan_;
};

// One run of n sequences of one length: every step but the last holds a multiple of `devices` sequences
// (dealt round-robin, so every sub-batch holds the same count), the last splits into q equal sub-batches;
// the fewest steps that fit cap = min(budget / len, n) sequences a sub-batch.
Plan fixed_length_plan(const Run& run, int64_t len, int64_t budget, int devices) {
    const int64_t n = (int64_t)run.size(), d = devices, cap = std::min<int64_t>(budget / len, n);
    const int64_t full = d * cap;
    int64_t steps = 0, tail = 0, tail_subs = 1;
    for (int64_t s = std::max<int64_t>(1, (n + full - 1) / full); steps == 0; ++s) {
        if (s == 1) {
            for (int64_t q = d; q >= 1; --q)
                if (n % q == 0 && n / q <= cap) {
                    steps = 1, tail = n, tail_subs = q;
                    break;
                }
            continue;
        }
        const int64_t min_body = (s - 1) * d, max_body = (s - 1) * full;
        for (int64_t q = d; q >= 1 && steps == 0; --q) {
            const int64_t low = std::max<int64_t>(q, n - max_body), high = std::min<int64_t>(q * cap, n - min_body);
            if (low > high) continue;
            const int64_t k_lo = std::max<int64_t>(1, (low + q - 1) / q), k_hi = std::min<int64_t>(cap, high / q);
            for (int64_t k = k_hi; k >= k_lo && k >= k_hi - d; --k)
                if ((q * k - n) % d == 0) {
                    steps = s, tail = q * k, tail_subs = q;
                    break;
                }
        }
    }
    Plan plan;
    size_t pos = 0;
    int64_t body = n - tail;
    for (int64_t i = 0; i + 1 < steps; ++i) {
        const int64_t after = steps - 2 - i;  // body steps still to come after this one
        const int64_t size = std::min(full, body - after * d) / d * d;
        Step step((size_t)d);
        for (int64_t j = 0; j < size; ++j) step[(size_t)(j % d)].push_back(run[pos + (size_t)j]);
        pos += (size_t)size;
        body -= size;
        plan.push_back(std::move(step));
    }
    Step last((size_t)tail_subs);
    for (int64_t j = 0; j < tail; ++j) last[(size_t)(j % tail_subs)].push_back(run[pos + (size_t)j]);
    plan.push_back(std::move(last));
    return plan;
}

// ------------------------------------------------------------------------------------------ batcher
struct Batcher {
    std::vector<int64_t> lens;
    int64_t budget = 0;
    int devices = 1;
    uint64_t seed = 0;
    std::vector<Index> skipped;
    int64_t skipped_tokens = 0;
    int64_t epoch = 0, step = 0;
    int64_t cached_epoch = -1;
    Plan cached;

    const Plan& plan(int64_t e) {
        if (cached_epoch == e) return cached;
        std::vector<Index> kept;
        kept.reserve(lens.size());
        size_t sk = 0;
        for (Index i = 0; i < (Index)lens.size(); ++i) {
            if (sk < skipped.size() && skipped[sk] == i) {
                ++sk;
                continue;
            }
            kept.push_back(i);
        }
        std::vector<Run> runs;
        for (Run& b : shuffled_buckets(std::move(kept), lens, seed, e)) {
            if (!runs.empty() && !b.empty() && length_class(lens[runs.back().front()]) == length_class(lens[b.front()]))
                runs.back().insert(runs.back().end(), b.begin(), b.end());
            else
                runs.push_back(std::move(b));
        }
        const bool fixed = runs.size() == 1 && !runs[0].empty() && lens[runs[0][0]] > 0 &&
                           std::all_of(runs[0].begin(), runs[0].end(),
                                       [&](Index i) { return lens[i] == lens[runs[0][0]]; });
        if (fixed) {
            cached = fixed_length_plan(runs[0], lens[runs[0][0]], budget, devices);
        } else {
            Packer p(lens, budget, devices);
            for (size_t i = 0; i < runs.size(); ++i) p.pack_run(runs[i], i + 1 < runs.size());
            cached = p.take();
        }
        cached_epoch = e;
        return cached;
    }
};

}  // namespace

extern "C" {

void* r97host_batcher_create(const int64_t* lengths, int64_t n, int64_t token_budget, int32_t devices,
                             uint64_t seed) {
    g_batcher_error.clear();
    if (token_budget <= 0) {
        g_batcher_error = "batcher: token_budget must be positive";
        return nullptr;
    }
    if (devices < 1) {
        g_batcher_error = "batcher: devices must be at least 1";
        return nullptr;
    }
    if (n < 0 || (n > 0 && !lengths)) {
        g_batcher_error = "batcher: no sequence lengths";
        return nullptr;
    }
    auto* b = new Batcher;
    b->lens.assign(lengths, lengths + n);
    b->budget = token_budget;
    b->devices = devices;
    b->seed = seed;
    for (int64_t i = 0; i < n; ++i) {
        if (b->lens[(size_t)i] < 0) {
            delete b;
            g_batcher_error = "batcher: negative sequence length";
            return nullptr;
        }
        if (b->lens[(size_t)i] > token_budget) {
            b->skipped.push_back(i);
            b->skipped_tokens += b->lens[(size_t)i];
        }
    }
    return b;
}

void r97host_batcher_destroy(void* h) { delete static_cast<Batcher*>(h); }

const char* r97host_batcher_error(void) { return g_batcher_error.c_str(); }

int64_t r97host_batcher_steps_in_epoch(void* h, int64_t epoch) {
    return (int64_t)static_cast<Batcher*>(h)->plan(epoch).size();
}

int32_t r97host_batcher_next(void* h, int64_t* counts, int64_t* indices, int64_t cap) {
    auto* b = static_cast<Batcher*>(h);
    const Plan& p = b->plan(b->epoch);
    if (b->step < 0 || b->step >= (int64_t)p.size()) {
        b->step = (int64_t)p.size();
        return 0;
    }
    const Step& st = p[(size_t)b->step];
    int64_t total = 0;
    for (const auto& sub : st) total += (int64_t)sub.size();
    if (total > cap) {
        g_batcher_error = "batcher: index buffer holds " + std::to_string(cap) + " of the step's " +
                          std::to_string(total) + " sequences";
        return -1;
    }
    int64_t o = 0;
    for (size_t d = 0; d < st.size(); ++d) {
        counts[d] = (int64_t)st[d].size();
        std::memcpy(indices + o, st[d].data(), st[d].size() * sizeof(int64_t));
        o += (int64_t)st[d].size();
    }
    ++b->step;
    return (int32_t)st.size();
}

void r97host_batcher_position(void* h, int64_t* epoch, int64_t* step) {
    const auto* b = static_cast<const Batcher*>(h);
    *epoch = b->epoch;
    *step = b->step;
}

void r97host_batcher_seek(void* h, int64_t epoch, int64_t step) {
    auto* b = static_cast<Batcher*>(h);
    b->epoch = std::max<int64_t>(epoch, 0);
    b->step = std::clamp<int64_t>(step, 0, (int64_t)b->plan(b->epoch).size());
}

void r97host_batcher_reset(void* h) {
    auto* b = static_cast<Batcher*>(h);
    b->epoch = 0;
    b->step = 0;
}

int64_t r97host_batcher_skipped(void* h, int64_t* out, int64_t cap) {
    const auto* b = static_cast<const Batcher*>(h);
    if (out)
        for (size_t i = 0; i < b->skipped.size() && (int64_t)i < cap; ++i) out[i] = b->skipped[i];
    return (int64_t)b->skipped.size();
}

int64_t r97host_batcher_skipped_tokens(void* h) { return static_cast<const Batcher*>(h)->skipped_tokens; }

}  // extern "C"
