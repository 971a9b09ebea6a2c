// The continuous-batching engine above the Kernel boundary: hk_engine_*.
//
// Behaviour follows the reference's engine module step for step, because the engine's
// observable output (the share stream it pushes, the tokens and ends each request hears, the
// metrics) is the contract a drop-in must keep:
//   Units / Cache          src/engine/cache.rs:46-359
//   Lane / Lanes           src/engine/lanes.rs:7-159
//   Clock                  src/engine/clock.rs:3-31
//   Plan / Pacing          src/engine/pacing.rs:1-61
//   StepMetrics / Hist     src/engine/metrics.rs:4-111
//   Request / Sampling     src/engine/request.rs:6-64
//   run / Engine           src/engine/mod.rs:38-359
// The kernel is reached only through hk_kernel_ops (hk_push / hk_drain semantics), so the same
// engine drives the device kernel (device.cu) or any other implementation of the trait.
#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "hk.h"

namespace hk {
int fail(int code, const char* fmt, ...);  // common.cu: sets hk_last_error()
void set_error(const std::string& msg) { fail(HK_OK, "%s", msg.c_str()); }
}  // namespace hk

namespace {

using u32 = uint32_t;
using u64 = uint64_t;

constexpr u64 kUsizeMax = UINT64_MAX;

u64 sat_add(u64 a, u64 b) { return a > kUsizeMax - b ? kUsizeMax : a + b; }
u64 sat_sub(u64 a, u64 b) { return a > b ? a - b : 0; }

// ---------------------------------------------------------------------------------------
// boundary values (src/gpu/mod.rs:13-40)
// ---------------------------------------------------------------------------------------

struct Sampled {
    int32_t id;
    std::vector<hk_logprob> logprobs;  // the reply's top pairs, then the token's own
};

struct Command {
    u32 kind = 0, lane = 0, pos = 0, upto = 0;  // pos = Pages.from / Seat.pos
    int32_t back[3] = {0, 0, 0};
    hk_sampling sampling{};
    std::vector<int32_t> data;  // Pages.row / Prompt.tokens
};

struct Share {
    u32 at, horizon;
    std::vector<Command> commands;
};

struct Event {
    u32 kind, step, lane;
    Sampled token;
    bool clipped;
    std::vector<std::vector<Sampled>> lanes;
};

bool nucleated(const hk_sampling& s) { return s.temperature > 0.0f && (s.top_p < 1.0f || s.top_k > 0); }

// ---------------------------------------------------------------------------------------
// requests and their output channels (src/engine/request.rs)
// ---------------------------------------------------------------------------------------

struct Out {
    u32 kind, end;  // a token's `end` is its logprob pair count
    int64_t value;
    std::string message;
    std::vector<hk_logprob> logprobs;
};

// Sender<Out>: a send fails once the listener hung up.
struct Sink {
    std::mutex m;
    std::condition_variable cv;
    std::deque<Out> items;
    bool listening = true;
    bool ended = false;

    bool send(Out o) {
        std::lock_guard<std::mutex> g(m);
        if (!listening) return false;
        if (o.kind == HK_OUT_END) ended = true;
        items.push_back(std::move(o));
        cv.notify_all();
        return true;
    }
};

struct Request {
    std::vector<u32> prompt;
    hk_sampling sampling{};
    u64 limit = 0;
    std::vector<u32> stop;
    std::shared_ptr<Sink> out;

    void took(u32 id) {
        prompt.push_back(id);
        limit -= 1;
    }
    u64 reach(u64 headroom, u64 context, u64 block) const {
        return std::min<u64>(prompt.size() + std::min(limit, headroom), context) + block - 1;
    }
};

enum class EndKind { Stop, Length, Refused };
struct End {
    EndKind kind;
    std::string message;
};

struct Job {
    bool reset = false;
    Request request;
    u64 ticket = 0;
};

// ---------------------------------------------------------------------------------------
// cache (src/engine/cache.rs)
// ---------------------------------------------------------------------------------------

struct Units {
    std::vector<u32> held;
    std::vector<u32> free;

    explicit Units(size_t n) : held(std::max<size_t>(n, 1), 0) {
        held[0] = 1;
        for (size_t u = n; u-- > 1;) free.push_back(static_cast<u32>(u));
    }
    std::optional<u32> take() {
        if (free.empty()) return std::nullopt;
        u32 u = free.back();
        free.pop_back();
        held[u] = 1;
        return u;
    }
    void share(u32 u) { held[u] += 1; }
    void release(u32 u) {
        if (--held[u] == 0) free.push_back(u);
    }
    bool once(u32 u) const { return held[u] == 1; }
};

struct Place {
    std::vector<u32> pages;
    std::vector<std::optional<u32>> window;
    u64 promise = 0, upto = 0;
    std::vector<int32_t> sent;
    u64 sent_upto = 0;
};

struct Node {
    std::optional<size_t> parent;
    std::vector<u32> tokens;
    u32 page;
    std::optional<u32> window;
    size_t children;
    u64 used;
};

struct EdgeKey {
    int64_t parent;  // -1 = the root
    std::vector<u32> tokens;
    bool operator==(const EdgeKey& o) const { return parent == o.parent && tokens == o.tokens; }
};
struct EdgeHash {
    size_t operator()(const EdgeKey& k) const {
        u64 h = 1469598103934665603ull ^ static_cast<u64>(k.parent);
        for (u32 t : k.tokens) h = (h ^ t) * 1099511628211ull;
        return static_cast<size_t>(h);
    }
};

struct WaitNever {
    std::string why;
};
struct WaitLater {};
struct HoldError {
    std::string why;
};

class Cache {
   public:
    Cache(const hk_engine_config& c, size_t pages, size_t window_pages, size_t lanes)
        : rows_(c.page_rows),
          entries_(c.entries),
          window_(c.window),
          keep_(c.window_keep > 0),
          pages_(pages),
          windows_(window_pages),
          lanes_(lanes) {
        for (auto& l : lanes_) l.sent.assign(entries_ + window_, 0);
    }

    // Ok(cached) or throws WaitLater / WaitNever (cache.rs:100-141)
    size_t admit(size_t lane, const std::vector<u32>& prompt, u64 extent) {
        const u64 p = rows_;
        extent = std::min<u64>(extent, entries_ * p);
        if (prompt.size() > extent)
            throw WaitNever{"a prompt of " + std::to_string(prompt.size()) + " tokens past a row's " +
                            std::to_string(entries_) + " pages of " + std::to_string(p)};
        std::vector<size_t> path = find(prompt);
        const u64 need = (extent + p - 1) / p - path.size();
        if (spare() + freeable(path) < static_cast<int64_t>(need)) {
            bool live = false;
            for (auto& l : lanes_) live |= !l.pages.empty() || l.promise > 0;
            if (!live || need + path.size() > pages_.held.size() - 1)
                throw WaitNever{std::to_string(need) + " pages more than its " + std::to_string(path.size()) +
                                " of a pool of " + std::to_string(pages_.held.size() - 1)};
            throw WaitLater{};
        }
        while (spare() < static_cast<int64_t>(need)) {
            if (!evict_page(path)) throw std::logic_error("admission counted pages the tree does not free");
        }
        const u64 now = tick();
        for (size_t n : path) {
            Node& node = nodes_.at(n);
            node.used = now;
            pages_.share(node.page);
            lanes_[lane].pages.push_back(node.page);
        }
        if (!path.empty()) {
            std::optional<u32> w = nodes_.at(path.back()).window;
            if (!w) throw std::logic_error("a resume's window page");
            windows_.share(*w);
            lanes_[lane].window.assign(path.size() - 1, std::nullopt);
            lanes_[lane].window.push_back(w);
        }
        lanes_[lane].promise = need;
        return path.size() * p;
    }

    // cache.rs:143-185; throws HoldError
    void hold(size_t lane, u64 start, u64 end) {
        const u64 p = rows_;
        const u64 last = (end - 1) / p;
        if (last >= entries_ || last >= window_)
            throw HoldError{"position " + std::to_string(end - 1) + " past a row's " +
                            std::to_string(std::min(entries_, window_)) + " pages of " + std::to_string(p)};
        while (lanes_[lane].pages.size() <= last) {
            Place& place = lanes_[lane];
            std::optional<u32> page;
            if (place.promise > 0) {
                place.promise -= 1;
                page = pages_.take();
            } else if (spare() > 0) {
                page = pages_.take();
            } else if (evict_page({})) {
                continue;
            } else {
                throw HoldError{"no page free"};
            }
            if (!page) throw std::logic_error("a free page");
            lanes_[lane].pages.push_back(*page);
        }
        const u64 from = sat_sub((start + 1) / p, 1);
        Place& place = lanes_[lane];
        for (size_t i = 0; i < std::min<size_t>(from, place.window.size()); ++i) {
            if (place.window[i]) {
                windows_.release(*place.window[i]);
                place.window[i].reset();
            }
        }
        if (place.window.size() <= last) place.window.resize(last + 1);
        for (u64 k = from; k <= last; ++k) {
            while (!lanes_[lane].window[k]) {
                if (std::optional<u32> w = windows_.take()) {
                    lanes_[lane].window[k] = w;
                } else if (!evict_window()) {
                    throw HoldError{"no window page free"};
                }
            }
        }
    }

    void run_to(size_t lane, u64 upto) { lanes_[lane].upto = upto; }
    u64 upto(size_t lane) const { return lanes_[lane].upto; }

    // cache.rs:195-226
    std::vector<Command> pages(size_t lane, u64 gap) {
        Place& place = lanes_[lane];
        std::vector<int32_t> row(entries_ + window_, 0);
        for (size_t k = 0; k < std::min<size_t>(place.pages.size(), entries_); ++k)
            row[k] = static_cast<int32_t>(place.pages[k]);
        for (size_t k = 0; k < std::min<size_t>(place.window.size(), window_); ++k)
            row[entries_ + k] = place.window[k] ? static_cast<int32_t>(*place.window[k]) : 0;
        std::vector<std::pair<size_t, size_t>> runs;
        for (size_t k = 0; k < row.size(); ++k) {
            if (row[k] == place.sent[k]) continue;
            if (!runs.empty() && k < runs.back().second + gap)
                runs.back().second = k + 1;
            else
                runs.emplace_back(k, k + 1);
        }
        if (runs.empty() && place.upto == place.sent_upto) return {};
        if (runs.empty()) runs.emplace_back(0, 0);
        std::vector<Command> out;
        for (auto [a, b] : runs) {
            Command c;
            c.kind = HK_CMD_PAGES;
            c.lane = static_cast<u32>(lane);
            c.pos = static_cast<u32>(a);
            c.upto = static_cast<u32>(place.upto);
            c.data.assign(row.begin() + a, row.begin() + b);
            out.push_back(std::move(c));
        }
        place.sent = std::move(row);
        place.sent_upto = place.upto;
        return out;
    }

    void finish(size_t lane, const std::vector<u32>& tokens, size_t len) {
        remember(lane, tokens, len);
        Place& place = lanes_[lane];
        for (u32 p : place.pages) pages_.release(p);
        place.pages.clear();
        for (auto& w : place.window)
            if (w) windows_.release(*w);
        place.window.clear();
        place.promise = place.upto = place.sent_upto = 0;
    }

    size_t pool() const { return pages_.held.size() - 1; }
    size_t held() const {
        size_t n = 0;
        for (auto& l : lanes_) n += l.pages.size();
        return n;
    }

    size_t reset() {
        const size_t free = pages_.free.size();
        std::map<size_t, Node> nodes;
        nodes.swap(nodes_);
        for (auto& [n, node] : nodes) {
            pages_.release(node.page);
            if (node.window) windows_.release(*node.window);
        }
        edges_.clear();
        return pages_.free.size() - free;
    }

   private:
    u64 tick() { return ++clock_; }

    int64_t spare() const {
        int64_t promised = 0;
        for (auto& l : lanes_) promised += static_cast<int64_t>(l.promise);
        return static_cast<int64_t>(pages_.free.size()) - promised;
    }

    std::vector<size_t> find(const std::vector<u32>& prompt) const {
        std::vector<size_t> path;
        size_t best = 0;
        int64_t parent = -1;
        const size_t r = rows_;
        for (size_t i = 0; i < prompt.size() / r; ++i) {
            if ((path.size() + 1) * r >= prompt.size()) break;
            EdgeKey key{parent, std::vector<u32>(prompt.begin() + i * r, prompt.begin() + (i + 1) * r)};
            auto it = edges_.find(key);
            if (it == edges_.end()) break;
            path.push_back(it->second);
            if (nodes_.at(it->second).window) best = path.size();
            parent = static_cast<int64_t>(it->second);
        }
        path.resize(best);
        return path;
    }

    static bool kept(const std::vector<size_t>& keep, size_t n) {
        return std::find(keep.begin(), keep.end(), n) != keep.end();
    }

    int64_t freeable(const std::vector<size_t>& keep) const {
        int64_t c = 0;
        for (auto& [n, node] : nodes_) c += !kept(keep, n) && pages_.once(node.page);
        return c;
    }

    template <class Pick>
    std::optional<size_t> lru(const std::vector<size_t>& keep, Pick pick) const {
        std::optional<size_t> best;
        u64 used = 0;
        for (auto& [n, node] : nodes_) {  // ascending ids: the first of equal `used` wins
            if (kept(keep, n) || !pick(node)) continue;
            if (!best || node.used < used) {
                best = n;
                used = node.used;
            }
        }
        return best;
    }

    bool evict_page(const std::vector<size_t>& keep) {
        auto n = lru(keep, [&](const Node& node) { return node.children == 0 && pages_.once(node.page); });
        if (!n) return false;
        Node node = std::move(nodes_.at(*n));
        nodes_.erase(*n);
        edges_.erase(EdgeKey{node.parent ? static_cast<int64_t>(*node.parent) : -1, node.tokens});
        if (node.parent) nodes_.at(*node.parent).children -= 1;
        pages_.release(node.page);
        if (node.window) windows_.release(*node.window);
        return true;
    }

    bool evict_window() {
        auto alone = [&](const Node& node) { return node.window && windows_.once(*node.window); };
        std::optional<size_t> n;
        if (keep_) n = lru({}, [&](const Node& node) { return alone(node) && node.children > 0; });
        if (!n) n = lru({}, alone);
        if (!n) return false;
        Node& node = nodes_.at(*n);
        u32 w = *node.window;
        node.window.reset();
        windows_.release(w);
        return true;
    }

    void remember(size_t lane, const std::vector<u32>& tokens, size_t len) {
        const u64 now = tick();
        std::optional<size_t> parent;
        const size_t r = rows_;
        for (size_t k = 0; k < len / r; ++k) {
            EdgeKey key{parent ? static_cast<int64_t>(*parent) : -1,
                        std::vector<u32>(tokens.begin() + k * r, tokens.begin() + (k + 1) * r)};
            size_t n;
            auto it = edges_.find(key);
            if (it != edges_.end()) {
                n = it->second;
            } else {
                if (k >= lanes_[lane].pages.size()) return;
                const u32 page = lanes_[lane].pages[k];
                pages_.share(page);
                n = ++ids_;
                nodes_.emplace(n, Node{parent, key.tokens, page, std::nullopt, 0, now});
                edges_.emplace(std::move(key), n);
                if (parent) nodes_.at(*parent).children += 1;
            }
            const auto& win = lanes_[lane].window;
            std::optional<u32> held = k < win.size() ? win[k] : std::nullopt;
            Node& node = nodes_.at(n);
            node.used = now;
            if (!node.window && held) {
                node.window = held;
                windows_.share(*held);
            }
            parent = n;
        }
    }

    size_t rows_, entries_, window_;
    bool keep_;
    Units pages_, windows_;
    std::vector<Place> lanes_;
    std::map<size_t, Node> nodes_;
    std::unordered_map<EdgeKey, size_t, EdgeHash> edges_;
    size_t ids_ = 0;
    u64 clock_ = 0;
};

// ---------------------------------------------------------------------------------------
// lanes (src/engine/lanes.rs)
// ---------------------------------------------------------------------------------------

struct Range {
    u64 start, end;
};

struct Lane {
    size_t lane;
    u64 seat;
    Request request;
    u64 sent;
    std::optional<u32> from;

    bool decoding() const { return from.has_value(); }
    bool decodes_at(u32 step) const { return from && step >= *from; }
    u64 written() const { return decoding() ? request.prompt.size() - 1 : sent; }

    Range next_chunk(u64 rows, u64 tokens) const {
        return {sent, sent + std::min({request.prompt.size() - sent, rows, tokens})};
    }

    std::vector<Command> chunk(Range piece, int32_t pad) const {
        const auto& toks = request.prompt;
        Command seat;
        seat.kind = HK_CMD_SEAT;
        seat.lane = static_cast<u32>(lane);
        seat.pos = static_cast<u32>(piece.start);
        for (int j = 0; j < 3; ++j)
            seat.back[j] = piece.start + j >= 3 ? static_cast<int32_t>(toks[piece.start + j - 3]) : pad;
        seat.sampling = request.sampling;
        Command prompt;
        prompt.kind = HK_CMD_PROMPT;
        prompt.lane = static_cast<u32>(lane);
        for (u64 i = piece.start; i < piece.end; ++i) prompt.data.push_back(static_cast<int32_t>(toks[i]));
        std::vector<Command> out{seat, prompt};
        if (piece.end == toks.size()) {
            Command start;
            start.kind = HK_CMD_START;
            start.lane = static_cast<u32>(lane);
            out.push_back(start);
        }
        return out;
    }

    std::optional<Range> ahead(u64 upto, u64 context, u64 block, u64 ahead) const {
        const u64 next = request.prompt.size() - 1;
        const u64 last = std::min(sat_add(request.prompt.size(), request.limit), context) - 2;
        const u64 end = std::min(next + ahead, last + 1) + block - 1;
        if (end > next + block - 1 && upto < end && upto < next + ahead / 2 + block) return Range{next, end};
        return std::nullopt;
    }

    std::optional<End> hear(const Sampled& t, u64 context) {
        if (t.id < 0) return End{EndKind::Refused, "the kernel's logits were not finite"};
        const u32 id = static_cast<u32>(t.id);
        Request& r = request;
        // the token's own pair, then the first `ask` of the top pairs (lanes.rs:58-64)
        std::vector<hk_logprob> lps;
        const u64 ask = r.sampling.logprobs;
        if (ask > 0 && !t.logprobs.empty()) {
            lps.push_back(t.logprobs.back());
            for (size_t i = 0; i + 1 < t.logprobs.size() && i < ask; ++i) lps.push_back(t.logprobs[i]);
        }
        const u32 n_lp = static_cast<u32>(lps.size());
        if (!r.out->send(Out{HK_OUT_TOKEN, n_lp, static_cast<int64_t>(id), {}, std::move(lps)}))
            return End{EndKind::Stop, {}};
        if (std::find(r.stop.begin(), r.stop.end(), id) != r.stop.end()) return End{EndKind::Stop, {}};
        r.took(id);
        if (r.limit == 0 || r.prompt.size() >= context) return End{EndKind::Length, {}};
        return std::nullopt;
    }
};

class Lanes {
   public:
    explicit Lanes(size_t width) : slots_(width) {}

    std::optional<size_t> free() const {
        for (size_t i = 0; i < slots_.size(); ++i)
            if (slots_[i].state == kFree) return i;
        return std::nullopt;
    }
    void seat(size_t lane, Request r, u64 cached) {
        seats_ += 1;
        slots_[lane].state = kHeld;
        slots_[lane].lane.reset(new Lane{lane, seats_, std::move(r), cached, std::nullopt});
    }
    Lane take(size_t lane) {
        if (slots_[lane].state != kHeld) throw std::logic_error("lane taken unheld");
        Lane l = std::move(*slots_[lane].lane);
        slots_[lane].lane.reset();
        slots_[lane].state = kEnding;
        return l;
    }
    std::vector<u32> ended() {
        std::vector<u32> out;
        for (size_t i = 0; i < slots_.size(); ++i) {
            if (slots_[i].state == kEnding) {
                slots_[i].state = kFree;
                out.push_back(static_cast<u32>(i));
            }
        }
        return out;
    }
    Lane* get(size_t lane) { return slots_[lane].state == kHeld ? slots_[lane].lane.get() : nullptr; }
    bool is_empty() const {
        for (auto& s : slots_)
            if (s.state != kFree) return false;
        return true;
    }
    template <class Pick>
    std::vector<size_t> by_seat(Pick pick) const {
        std::vector<const Lane*> ls;
        for (auto& s : slots_)
            if (s.state == kHeld && pick(*s.lane)) ls.push_back(s.lane.get());
        std::sort(ls.begin(), ls.end(), [](const Lane* a, const Lane* b) { return a->seat < b->seat; });
        std::vector<size_t> out;
        for (auto* l : ls) out.push_back(l->lane);
        return out;
    }
    std::vector<size_t> held() const { return by_seat([](const Lane&) { return true; }); }
    std::vector<size_t> prompting() const { return by_seat([](const Lane& l) { return !l.decoding(); }); }
    std::vector<size_t> decoding() const { return by_seat([](const Lane& l) { return l.decoding(); }); }
    std::optional<size_t> newest() const {
        auto h = held();
        if (h.empty()) return std::nullopt;
        return h.back();
    }

   private:
    enum { kFree, kHeld, kEnding };
    struct Slot {
        int state = kFree;
        std::unique_ptr<Lane> lane;
    };
    std::vector<Slot> slots_;
    u64 seats_ = 0;
};

// ---------------------------------------------------------------------------------------
// clock, pacing, metrics
// ---------------------------------------------------------------------------------------

class Clock {
   public:
    explicit Clock(u32 lead) : lead_(lead) {}
    void saw(u32 step) { seen_ = step; }
    u32 next() const { return granted_; }
    std::optional<Share> grant(std::vector<Command> commands, bool decoding) {
        const bool running_out = seen_ + lead_ >= granted_;
        if (commands.empty() && !(decoding && running_out)) return std::nullopt;
        const u32 at = granted_;
        const u32 from = commands.empty() ? seen_ : std::max(seen_, at > 0 ? at - 1 : 0);
        granted_ = from + lead_ + 1;
        return Share{at, from + lead_, std::move(commands)};
    }

   private:
    u32 lead_, seen_ = 0, granted_ = 0;
};

struct Allowance {
    u64 chunks, tokens;
    bool left() const { return chunks > 0 && tokens > 0; }
    void spend(u64 n) {
        chunks -= 1;
        tokens -= n;
    }
};

class Pacing {
   public:
    Pacing(u64 budget, u64 every, u64 headroom) : budget_(budget), every_(every), headroom_(headroom) {}
    bool due(size_t decoding) const { return decoding == 0 || steps_ + 1 >= every_; }
    Allowance allowance(size_t decoding, u64 block) const {
        if (budget_ == HK_UNBOUNDED) return {1, kUsizeMax};
        return {kUsizeMax, sat_sub(budget_, decoding * block)};
    }
    u64 headroom() const { return headroom_; }
    void stepped() { steps_ += 1; }
    void prefilled() { steps_ = 0; }

   private:
    u64 budget_, every_, headroom_, steps_ = 0;
};

struct StepMetrics {
    hk_step_metrics m{};
    std::vector<u64> accepted_per_pos;

    StepMetrics then(const StepMetrics& n) const {
        StepMetrics s;
        s.m = n.m;
        s.m.prompt_tokens = m.prompt_tokens + n.m.prompt_tokens;
        s.m.cached_tokens = m.cached_tokens + n.m.cached_tokens;
        s.m.prefill_tokens = m.prefill_tokens + n.m.prefill_tokens;
        s.m.generation_tokens = m.generation_tokens + n.m.generation_tokens;
        s.m.preemptions = m.preemptions + n.m.preemptions;
        s.m.top_p_clipped = m.top_p_clipped + n.m.top_p_clipped;
        s.m.drafts = m.drafts + n.m.drafts;
        const size_t len = std::max(accepted_per_pos.size(), n.accepted_per_pos.size());
        s.accepted_per_pos.resize(len, 0);
        for (size_t i = 0; i < len; ++i)
            s.accepted_per_pos[i] = (i < accepted_per_pos.size() ? accepted_per_pos[i] : 0) +
                                    (i < n.accepted_per_pos.size() ? n.accepted_per_pos[i] : 0);
        return s;
    }
    void verified(size_t accepted) {
        m.drafts += 1;
        if (accepted_per_pos.size() < accepted) accepted_per_pos.resize(accepted, 0);
        for (size_t i = 0; i < accepted; ++i) accepted_per_pos[i] += 1;
    }
    u64 tokens() const { return m.prefill_tokens + m.generation_tokens; }
};

// Metrics with the default iteration_tokens bounds of the reference's metrics config.
class Metrics {
   public:
    static constexpr double kBounds[13] = {1, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384};

    void record(const StepMetrics& step) {
        std::lock_guard<std::mutex> g(m_);
        if (step.tokens() > 0) {
            const double x = static_cast<double>(step.tokens());
            size_t i = 0;
            while (i < 13 && kBounds[i] < x) ++i;
            counts_[i] += 1;
            sum_ += x;
        }
        total_ = total_.then(step);
    }
    void read(StepMetrics* total, u64 counts[14], double* sum) {
        std::lock_guard<std::mutex> g(m_);
        *total = total_;
        std::copy(counts_, counts_ + 14, counts);
        *sum = sum_;
    }

   private:
    std::mutex m_;
    StepMetrics total_;
    u64 counts_[14] = {};
    double sum_ = 0;
};

// ---------------------------------------------------------------------------------------
// the kernel seen through hk_kernel_ops
// ---------------------------------------------------------------------------------------

struct KernelError {
    int code;
    std::string message;
};

class KernelPort {
   public:
    KernelPort(const hk_kernel_ops& ops, size_t width, size_t block) : ops_(ops), width_(width), block_(block) {}

    std::pair<size_t, size_t> pools() {
        size_t p = 0, w = 0;
        check(ops_.pools(ops_.self, &p, &w));
        return {p, w};
    }

    void push(const Share& s) {
        std::vector<hk_command> cmds;
        std::vector<int32_t> arena;
        cmds.reserve(s.commands.size());
        for (const Command& c : s.commands) {
            hk_command h{};
            h.kind = c.kind;
            h.lane = c.lane;
            h.pos = c.pos;
            h.upto = c.upto;
            h.count = static_cast<u32>(c.data.size());
            h.arena = static_cast<u32>(arena.size());
            std::copy(c.back, c.back + 3, h.back);
            h.sampling = c.sampling;
            arena.insert(arena.end(), c.data.begin(), c.data.end());
            cmds.push_back(h);
        }
        hk_share hs{s.at, s.horizon, cmds.data(), cmds.size(), arena.data(), arena.size()};
        check(ops_.push(ops_.self, &hs));
    }

    std::vector<Event> drain() {
        size_t n = 0, ids_n = 0;
        for (;;) {
            int rc = ops_.drain(ops_.self, events_.data(), events_.size(), &n, ids_.data(), ids_.size(), &ids_n);
            if (rc == HK_ESPACE) {
                events_.resize(std::max(n, events_.size() * 2 + 16));
                ids_.resize(std::max(ids_n, ids_.size() * 2 + 64));
                continue;
            }
            check(rc);
            break;
        }
        // the logprob lists, one per Sampled slot in event order (none without the callback)
        size_t n_lists = 0, n_pairs = 0;
        if (ops_.logprobs) {
            for (;;) {
                int rc = ops_.logprobs(ops_.self, counts_.data(), counts_.size(), &n_lists, pairs_.data(),
                                       pairs_.size(), &n_pairs);
                if (rc == HK_ESPACE) {
                    counts_.resize(std::max(n_lists, counts_.size() * 2 + 64));
                    pairs_.resize(std::max(n_pairs, pairs_.size() * 2 + 64));
                    continue;
                }
                check(rc);
                break;
            }
        }
        size_t list = 0, pair = 0;
        auto take = [&](Sampled& smp) {  // the next list, attached to `smp` when it is a sampled value
            if (!ops_.logprobs) return;
            if (list >= n_lists) throw KernelError{HK_EINVAL, "fewer logprob lists than sampled slots"};
            const u32 c = counts_[list++];
            if (pair + c > n_pairs) throw KernelError{HK_EINVAL, "logprob pairs past the drained pairs"};
            smp.logprobs.assign(pairs_.begin() + pair, pairs_.begin() + pair + c);
            pair += c;
        };
        std::vector<Event> out;
        out.reserve(n);
        for (size_t i = 0; i < n; ++i) {
            const hk_event& e = events_[i];
            Event ev{e.kind, e.step, e.lane, Sampled{e.token, {}}, e.clipped != 0, {}};
            if (e.kind == HK_EV_STEP) {
                if (e.ids + width_ * block_ > ids_n) throw KernelError{HK_EINVAL, "a step's ids past the drained ids"};
                ev.lanes.resize(width_);
                for (size_t l = 0; l < width_; ++l) {
                    bool open = true;  // a lane's list ends at its first -2
                    for (size_t k = 0; k < block_; ++k) {
                        const int32_t id = ids_[e.ids + l * block_ + k];
                        Sampled smp{id, {}};
                        take(smp);
                        if (id == -2) open = false;
                        if (open) ev.lanes[l].push_back(std::move(smp));
                    }
                }
            } else if (e.kind == HK_EV_PROMPTED) {
                take(ev.token);
            }
            out.push_back(std::move(ev));
        }
        if (ops_.logprobs && list != n_lists) throw KernelError{HK_EINVAL, "more logprob lists than sampled slots"};
        return out;
    }

   private:
    void check(int rc) {
        if (rc == HK_OK) return;
        const char* msg = ops_.error ? ops_.error(ops_.self) : nullptr;
        throw KernelError{rc, msg ? msg : "the kernel failed"};
    }
    hk_kernel_ops ops_;
    size_t width_, block_;
    std::vector<hk_event> events_ = std::vector<hk_event>(64);
    std::vector<int32_t> ids_ = std::vector<int32_t>(1024);
    std::vector<uint32_t> counts_ = std::vector<uint32_t>(1024);
    std::vector<hk_logprob> pairs_ = std::vector<hk_logprob>(1024);
};

// ---------------------------------------------------------------------------------------
// the job channel (std::sync::mpsc semantics)
// ---------------------------------------------------------------------------------------

class Jobs {
   public:
    enum class Got { Job, Empty, Closed };

    void send(Job j) {
        std::lock_guard<std::mutex> g(m_);
        q_.push_back(std::move(j));
        cv_.notify_all();
    }
    void close() {
        std::lock_guard<std::mutex> g(m_);
        closed_ = true;
        cv_.notify_all();
    }
    Got try_recv(Job* j) {
        std::lock_guard<std::mutex> g(m_);
        if (!q_.empty()) {
            *j = std::move(q_.front());
            q_.pop_front();
            return Got::Job;
        }
        return closed_ ? Got::Closed : Got::Empty;
    }
    Got recv(Job* j) {
        std::unique_lock<std::mutex> g(m_);
        cv_.wait(g, [&] { return !q_.empty() || closed_; });
        if (q_.empty()) return Got::Closed;
        *j = std::move(q_.front());
        q_.pop_front();
        return Got::Job;
    }
    std::vector<Job> drain() {
        std::lock_guard<std::mutex> g(m_);
        std::vector<Job> out(std::make_move_iterator(q_.begin()), std::make_move_iterator(q_.end()));
        q_.clear();
        return out;
    }

   private:
    std::mutex m_;
    std::condition_variable cv_;
    std::deque<Job> q_;
    bool closed_ = false;
};

// ---------------------------------------------------------------------------------------
// the engine (src/engine/mod.rs:76-359)
// ---------------------------------------------------------------------------------------

struct Asked {
    size_t lane;
    u64 seat;
    bool last, nucleated;
};

struct ResetAnswers {
    std::mutex m;
    std::condition_variable cv;
    std::unordered_map<u64, u64> freed;
};

class Engine {
   public:
    Engine(const hk_engine_config& c, std::pair<size_t, size_t> pools, ResetAnswers* answers)
        : c_(c),
          lanes_(c.width),
          cache_(c, pools.first, pools.second, c.width),
          clock_(c.lead),
          pacing_(c.budget, c.every, c.headroom),
          answers_(answers) {}

    bool take(Jobs& jobs) {
        for (;;) {
            Job j;
            Jobs::Got g = jobs.try_recv(&j);
            if (g == Jobs::Got::Empty) break;
            if (g == Jobs::Got::Closed) return !idle();
            job(std::move(j));
        }
        if (idle()) {
            Job j;
            if (jobs.recv(&j) == Jobs::Got::Closed) return false;
            job(std::move(j));
        }
        return true;
    }

    std::optional<Share> schedule() {
        extend_decodes();
        std::vector<Command> prompts = prefill();
        std::vector<Command> commands;
        for (u32 lane : lanes_.ended()) {
            Command e;
            e.kind = HK_CMD_END;
            e.lane = lane;
            commands.push_back(std::move(e));
        }
        for (size_t lane : lanes_.held()) {
            auto p = cache_.pages(lane, c_.gap);
            std::move(p.begin(), p.end(), std::back_inserter(commands));
        }
        std::move(prompts.begin(), prompts.end(), std::back_inserter(commands));
        return clock_.grant(std::move(commands), !lanes_.decoding().empty());
    }

    void hear(const Event& e) {
        if (e.kind == HK_EV_IDLE) {
            clock_.saw(e.step);
        } else if (e.kind == HK_EV_STEP) {
            clock_.saw(e.step);
            pacing_.stepped();
            for (size_t lane = 0; lane < e.lanes.size(); ++lane) decoded(lane, e.step, e.lanes[lane]);
        } else {
            prompted(e.lane, e.token, e.clipped);
        }
    }

    StepMetrics step_metrics() {
        StepMetrics s = std::move(step_);
        step_ = StepMetrics{};
        s.m.running = lanes_.held().size();
        s.m.waiting = waiting_.size();
        s.m.held_pages = cache_.held();
        s.m.pages = cache_.pool();
        s.m.spec_tokens = c_.block - 1;
        return s;
    }

    void refuse(const std::string& why, Jobs& jobs) {
        for (size_t lane : lanes_.held()) end(lane, End{EndKind::Refused, why});
        for (Request& r : waiting_) r.out->send(Out{HK_OUT_END, HK_END_REFUSED, 0, why});
        waiting_.clear();
        for (Job& j : jobs.drain())
            if (!j.reset) j.request.out->send(Out{HK_OUT_END, HK_END_REFUSED, 0, why});
    }

   private:
    void job(Job j) {
        if (!j.reset) {
            waiting_.push_back(std::move(j.request));
            return;
        }
        const u64 freed = cache_.reset();
        std::lock_guard<std::mutex> g(answers_->m);
        answers_->freed[j.ticket] = freed;
        answers_->cv.notify_all();
    }

    bool idle() const { return lanes_.is_empty() && waiting_.empty() && asked_.empty(); }

    void extend_decodes() {
        for (size_t lane : lanes_.decoding()) {
            Lane* l = lanes_.get(lane);
            if (!l) continue;
            auto rows = l->ahead(cache_.upto(lane), c_.context, c_.block, c_.ahead);
            if (!rows) continue;
            if (cover(lane, *rows)) cache_.run_to(lane, rows->end);
        }
    }

    std::vector<Command> prefill() {
        std::vector<size_t> seated = seat_waiting();
        const bool due = pacing_.due(lanes_.decoding().size());
        std::vector<Command> chunks_out = chunks(due ? lanes_.prompting() : seated);
        if (due && !chunks_out.empty()) pacing_.prefilled();
        return chunks_out;
    }

    std::vector<size_t> seat_waiting() {
        const u64 context = c_.context;
        std::vector<size_t> seated;
        for (;;) {
            std::optional<size_t> lane = lanes_.free();
            if (!lane || waiting_.empty()) return seated;
            Request& r = waiting_.front();
            const size_t n = r.prompt.size();
            End end;
            if (n == 0) {
                end = End{EndKind::Refused, "an empty prompt"};
            } else if (n >= context) {
                end = End{EndKind::Refused, "a prompt of " + std::to_string(n) + " tokens: the context holds " +
                                                std::to_string(context) + ", a token past it"};
            } else if (r.limit == 0) {
                end = End{EndKind::Length, {}};
            } else {
                try {
                    const size_t cached =
                        cache_.admit(*lane, r.prompt, r.reach(pacing_.headroom(), context, c_.block));
                    seat(*lane, cached);
                    seated.push_back(*lane);
                    continue;
                } catch (const WaitLater&) {
                    return seated;
                } catch (const WaitNever& w) {
                    end = End{EndKind::Refused, "the cache: " + w.why};
                }
            }
            Request gone = std::move(waiting_.front());
            waiting_.pop_front();
            send_end(gone, end);
        }
    }

    std::vector<Command> chunks(const std::vector<size_t>& lanes) {
        const u32 at = clock_.next();
        Allowance allowance = pacing_.allowance(lanes_.decoding().size(), c_.block);
        std::vector<Command> out;
        for (size_t lane : lanes) {
            if (!allowance.left()) break;
            Lane* l = lanes_.get(lane);
            if (!l) continue;
            const Range piece = l->next_chunk(c_.chunk, allowance.tokens);
            const bool last = piece.end == l->request.prompt.size();
            std::optional<Range> ahead;
            if (last) ahead = l->ahead(cache_.upto(lane), c_.context, c_.block, c_.ahead);
            if (!cover(lane, piece) || (ahead && !cover(lane, Range{piece.start, ahead->end}))) continue;
            if (ahead) cache_.run_to(lane, ahead->end);
            l = lanes_.get(lane);
            auto cmds = l->chunk(piece, c_.pad);
            std::move(cmds.begin(), cmds.end(), std::back_inserter(out));
            l->sent = piece.end;
            if (last) l->from = at;
            asked_.push_back(Asked{lane, l->seat, last, nucleated(l->request.sampling)});
            step_.m.prefill_tokens += piece.end - piece.start;
            allowance.spend(piece.end - piece.start);
        }
        return out;
    }

    bool cover(size_t lane, Range rows) {
        for (;;) {
            try {
                cache_.hold(lane, rows.start, rows.end);
                return true;
            } catch (const HoldError& e) {
                std::optional<size_t> newest = lanes_.newest();
                if (!newest) throw std::logic_error("a held lane");
                if (lanes_.held().size() == 1) {
                    end(lane, End{EndKind::Refused, "the cache: " + e.why});
                    return false;
                }
                preempt(*newest);
                if (*newest == lane) return false;
            }
        }
    }

    void prompted(size_t lane, Sampled token, bool clipped) {
        if (asked_.empty()) throw KernelError{HK_ESTATE, "a prompt chunk's reply with no chunk asked"};
        Asked asked = asked_.front();
        asked_.pop_front();
        if (asked.lane != lane) throw KernelError{HK_ESTATE, "a prompt chunk's reply for another lane"};
        step_.m.top_p_clipped += clipped && asked.nucleated;
        Lane* l = lanes_.get(lane);
        if (asked.last && l && l->seat == asked.seat) heard(lane, token);
    }

    void decoded(size_t lane, u32 step, const std::vector<Sampled>& tokens) {
        Lane* l = lanes_.get(lane);
        if (!l || !l->decodes_at(step)) return;
        if (c_.block > 1 && !tokens.empty() &&
            std::all_of(tokens.begin(), tokens.end(), [](const Sampled& t) { return t.id >= 0; }))
            step_.verified(tokens.size() - 1);
        for (const Sampled& t : tokens)
            if (!heard(lane, t)) return;
    }

    bool heard(size_t lane, Sampled t) {
        step_.m.generation_tokens += 1;
        std::optional<End> e = lanes_.get(lane)->hear(t, c_.context);
        if (e) end(lane, *e);
        return !e;
    }

    void seat(size_t lane, size_t cached) {
        Request r = std::move(waiting_.front());
        waiting_.pop_front();
        step_.m.prompt_tokens += r.prompt.size();
        step_.m.cached_tokens += cached;
        r.out->send(Out{HK_OUT_SEATED, 0, static_cast<int64_t>(cached), {}});
        lanes_.seat(lane, std::move(r), cached);
    }

    void preempt(size_t lane) {
        step_.m.preemptions += 1;
        waiting_.push_front(free(lane));
    }

    void end(size_t lane, const End& why) {
        Request r = free(lane);
        send_end(r, why);
    }

    static void send_end(Request& r, const End& why) {
        const u32 kind = why.kind == EndKind::Stop ? HK_END_STOP
                         : why.kind == EndKind::Length ? HK_END_LENGTH
                                                       : HK_END_REFUSED;
        r.out->send(Out{HK_OUT_END, kind, 0, why.message});
    }

    Request free(size_t lane) {
        Lane l = lanes_.take(lane);
        cache_.finish(lane, l.request.prompt, l.written());
        return std::move(l.request);
    }

    hk_engine_config c_;
    std::deque<Request> waiting_;
    Lanes lanes_;
    Cache cache_;
    std::deque<Asked> asked_;
    Clock clock_;
    Pacing pacing_;
    StepMetrics step_;
    ResetAnswers* answers_;
};

}  // namespace

struct hk_engine {
    hk_engine_config config;
    hk_kernel_ops ops;
    Jobs jobs;
    Metrics metrics;
    ResetAnswers answers;
    std::mutex m;
    std::unordered_map<u64, std::shared_ptr<Sink>> sinks;
    u64 next_request = 1, next_ticket = 1;
};

extern "C" {

void hk_engine_defaults(hk_engine_config* c) {
    if (!c) return;
    std::memset(c, 0, sizeof(*c));
    c->budget = HK_UNBOUNDED;
    c->every = 1;
    c->headroom = 2048;
    c->gap = 16;
    c->lead = 2;
    c->ahead = 16;
    c->max_draft_positions = 16;
    c->block = 1;
}

int hk_engine_create(const hk_engine_config* c, const hk_kernel_ops* kernel, hk_engine** engine) {
    if (!c || !kernel || !engine || !kernel->pools || !kernel->push || !kernel->drain) {
        hk::set_error("hk_engine_create: null config, kernel or callback");
        return HK_EINVAL;
    }
    if (c->page_rows == 0 || c->width == 0 || c->block == 0 || c->chunk == 0 || c->context < 2) {
        hk::set_error("hk_engine_create: page_rows, width, block, chunk must be > 0 and context >= 2");
        return HK_EINVAL;
    }
    if (c->block - 1 > c->max_draft_positions) {
        hk::set_error(std::to_string(c->block - 1) + " drafts a step, past the " +
                      std::to_string(c->max_draft_positions) + " the metrics count");
        return HK_EINVAL;
    }
    auto* e = new hk_engine;
    e->config = *c;
    e->ops = *kernel;
    *engine = e;
    return HK_OK;
}

void hk_engine_destroy(hk_engine* e) { delete e; }

int hk_engine_submit(hk_engine* e, const uint32_t* prompt, size_t n, const hk_sampling* s, uint64_t limit,
                     const uint32_t* stop, size_t n_stop, uint64_t* request) {
    if (!e || (n && !prompt) || (n_stop && !stop) || !request) {
        hk::set_error("hk_engine_submit: null argument");
        return HK_EINVAL;
    }
    Job j;
    j.request.prompt.assign(prompt, prompt + n);
    if (s) j.request.sampling = *s;
    j.request.limit = limit;
    j.request.stop.assign(stop, stop + n_stop);
    j.request.out = std::make_shared<Sink>();
    {
        std::lock_guard<std::mutex> g(e->m);
        *request = e->next_request++;
        e->sinks[*request] = j.request.out;
    }
    e->jobs.send(std::move(j));
    return HK_OK;
}

int hk_engine_reset(hk_engine* e, uint64_t* ticket) {
    if (!e || !ticket) {
        hk::set_error("hk_engine_reset: null argument");
        return HK_EINVAL;
    }
    Job j;
    j.reset = true;
    {
        std::lock_guard<std::mutex> g(e->m);
        j.ticket = *ticket = e->next_ticket++;
    }
    e->jobs.send(std::move(j));
    return HK_OK;
}

int hk_engine_reset_answer(hk_engine* e, uint64_t ticket, int64_t timeout_ms, uint64_t* freed) {
    if (!e || !freed) {
        hk::set_error("hk_engine_reset_answer: null argument");
        return HK_EINVAL;
    }
    std::unique_lock<std::mutex> g(e->answers.m);
    auto ready = [&] { return e->answers.freed.count(ticket) > 0; };
    if (timeout_ms < 0)
        e->answers.cv.wait(g, ready);
    else if (!e->answers.cv.wait_for(g, std::chrono::milliseconds(timeout_ms), ready)) {
        hk::set_error("hk_engine_reset_answer: no answer yet");
        return HK_ESTATE;
    }
    *freed = e->answers.freed[ticket];
    e->answers.freed.erase(ticket);
    return HK_OK;
}

int hk_engine_close(hk_engine* e) {
    if (!e) return HK_EINVAL;
    e->jobs.close();
    return HK_OK;
}

int hk_engine_hangup(hk_engine* e, uint64_t request) {
    if (!e) return HK_EINVAL;
    std::shared_ptr<Sink> s;
    {
        std::lock_guard<std::mutex> g(e->m);
        auto it = e->sinks.find(request);
        if (it == e->sinks.end()) {
            hk::set_error("hk_engine_hangup: no such request");
            return HK_EINVAL;
        }
        s = it->second;
    }
    std::lock_guard<std::mutex> g(s->m);
    s->listening = false;
    return HK_OK;
}

int hk_engine_run(hk_engine* e) {
    if (!e) return HK_EINVAL;
    const hk_engine_config& c = e->config;
    KernelPort kernel(e->ops, c.width, c.block);
    std::optional<Engine> engine;
    KernelError failure{HK_OK, {}};
    try {
        engine.emplace(c, kernel.pools(), &e->answers);
        e->metrics.record(engine->step_metrics());
        for (;;) {
            if (!engine->take(e->jobs)) return HK_OK;
            if (std::optional<Share> share = engine->schedule()) kernel.push(*share);
            for (const Event& ev : kernel.drain()) engine->hear(ev);
            e->metrics.record(engine->step_metrics());
        }
    } catch (const KernelError& k) {
        failure = k;
    } catch (const std::exception& x) {
        failure = KernelError{HK_ESTATE, std::string("engine invariant: ") + x.what()};
    }
    if (engine) {
        engine->refuse(failure.message, e->jobs);
        e->metrics.record(engine->step_metrics());
    }
    hk::set_error(failure.message);
    return failure.code;
}

int hk_engine_outputs_lp(hk_engine* e, uint64_t request, int64_t timeout_ms, hk_out* out, size_t cap, size_t* n,
                         char* message, size_t message_cap, hk_logprob* pairs, size_t pairs_cap, size_t* n_pairs) {
    if (!e || !n || (cap && !out) || (pairs && !n_pairs)) {
        hk::set_error("hk_engine_outputs: null argument");
        return HK_EINVAL;
    }
    std::shared_ptr<Sink> s;
    {
        std::lock_guard<std::mutex> g(e->m);
        auto it = e->sinks.find(request);
        if (it == e->sinks.end()) {
            hk::set_error("hk_engine_outputs: no such request");
            return HK_EINVAL;
        }
        s = it->second;
    }
    std::unique_lock<std::mutex> g(s->m);
    auto ready = [&] { return !s->items.empty(); };
    if (timeout_ms < 0)
        s->cv.wait(g, ready);
    else if (timeout_ms > 0)
        s->cv.wait_for(g, std::chrono::milliseconds(timeout_ms), ready);
    size_t k = 0, np = 0;
    while (k < cap && !s->items.empty()) {
        Out& o = s->items.front();
        if (pairs && np + o.logprobs.size() > pairs_cap) {  // never split a token's pairs
            if (k == 0) {
                *n = 0;
                *n_pairs = o.logprobs.size();
                hk::set_error("hk_engine_outputs_lp: pairs buffer too small");
                return HK_ESPACE;
            }
            break;
        }
        out[k++] = hk_out{o.kind, o.end, o.value};
        if (pairs) {
            std::copy(o.logprobs.begin(), o.logprobs.end(), pairs + np);
            np += o.logprobs.size();
        }
        if (o.kind == HK_OUT_END && message && message_cap) {
            const size_t len = std::min(o.message.size(), message_cap - 1);
            std::memcpy(message, o.message.data(), len);
            message[len] = 0;
        }
        s->items.pop_front();
    }
    *n = k;
    if (n_pairs) *n_pairs = np;
    return HK_OK;
}

int hk_engine_outputs(hk_engine* e, uint64_t request, int64_t timeout_ms, hk_out* out, size_t cap, size_t* n,
                      char* message, size_t message_cap) {
    return hk_engine_outputs_lp(e, request, timeout_ms, out, cap, n, message, message_cap, nullptr, 0, nullptr);
}

int hk_engine_metrics(hk_engine* e, hk_step_metrics* total, uint64_t* accepted_per_pos, size_t pos_cap,
                      size_t* n_pos, uint64_t* counts, size_t counts_cap, double* sum) {
    if (!e) return HK_EINVAL;
    StepMetrics t;
    u64 c[14];
    double s = 0;
    e->metrics.read(&t, c, &s);
    if (total) *total = t.m;
    if (n_pos) *n_pos = t.accepted_per_pos.size();
    if (accepted_per_pos)
        std::copy(t.accepted_per_pos.begin(), t.accepted_per_pos.begin() + std::min(pos_cap, t.accepted_per_pos.size()),
                  accepted_per_pos);
    if (counts) std::copy(c, c + std::min<size_t>(counts_cap, 14), counts);
    if (sum) *sum = s;
    return HK_OK;
}

}  // extern "C"
