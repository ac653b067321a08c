// The frame-slice scheduler: which slices run in a frame and when each
// result is delivered, the reference's Scheduler
// (crates/beatlm-core/src/schedule.rs:160-790) with its sync policies
// (sync.rs), frame budget (budget.rs) and beat grids (time.rs:140-330). It
// plans with the cost model's planning estimates, which this library feeds
// from cudaEvent timings. Host code only; a pure function of the frames,
// budgets and estimates it is given, so the rules are kept exactly as the
// reference states them (jobs run as one sequence, deadlines fixed at
// submission, a late job abandoned only when another waits behind it).
#include <algorithm>
#include <vector>

#include "host.h"

namespace bl {
namespace sched {

uint64_t sat_add(uint64_t a, uint64_t b) { return a > UINT64_MAX - b ? UINT64_MAX : a + b; }
uint64_t sat_sub(uint64_t a, uint64_t b) { return a > b ? a - b : 0; }
uint64_t sat_mul(uint64_t a, uint64_t b) {
    if (a == 0 || b == 0) return 0;
    return a > UINT64_MAX / b ? UINT64_MAX : a * b;
}

// BeatGrid::next_beat_at_or_after (time.rs): the origin for an instant at or
// before it, else the instant rounded up to the grid (saturating).
uint64_t grid_next(uint64_t origin, uint64_t beat, uint64_t t) {
    if (t <= origin) return origin;
    const uint64_t into = (t - origin) % beat;
    return into == 0 ? t : sat_add(t, beat - into);
}

struct Grid {
    uint64_t from, origin, beat;
};

// BeatMap (time.rs): grids in effect from increasing instants.
struct BeatMap {
    std::vector<Grid> grids;

    size_t in_effect(uint64_t t) const {  // the last grid whose `from` <= t
        size_t n = 0;
        while (n < grids.size() && grids[n].from <= t) ++n;
        return n > 0 ? n - 1 : 0;
    }
    void replace_from(uint64_t from, uint64_t origin, uint64_t beat) {
        grids.erase(std::remove_if(grids.begin(), grids.end(),
                                   [&](const Grid& g) { return g.from >= from; }),
                    grids.end());
        grids.push_back({from, origin, beat});
    }
    uint64_t next(uint64_t t) const {
        for (size_t i = in_effect(t); i < grids.size(); ++i) {
            const uint64_t b = grid_next(grids[i].origin, grids[i].beat, std::max(t, grids[i].from));
            // a beat that falls where the next grid is in effect: that one decides
            if (i + 1 < grids.size() && b >= grids[i + 1].from) {
                t = grids[i + 1].from;
                continue;
            }
            return b;
        }
        return t;
    }
    void forget_before(uint64_t t) { grids.erase(grids.begin(), grids.begin() + in_effect(t)); }
};

struct Due {
    bool beat;    // false: a frame index
    uint64_t at;  // the frame index, or the beat's instant

    bool reached(const bl_frame_info& f) const { return beat ? f.start_us >= at : f.index >= at; }
    bool on_time(const bl_frame_info& f) const {
        if (!beat) return f.index == at;
        return f.start_us == at || (f.start_us > at && f.start_us - at < f.period_us);
    }
    // frames from `f` to the one that keeps the deadline; false when behind
    bool frames_left(const bl_frame_info& f, uint64_t* left) const {
        if (!beat) {
            if (at < f.index) return false;
            *left = at - f.index;
            return true;
        }
        if (at <= f.start_us) {
            if (!on_time(f)) return false;
            *left = 0;
            return true;
        }
        const uint64_t ahead = at - f.start_us;
        *left = f.period_us == 0 ? UINT64_MAX : ahead / f.period_us + (ahead % f.period_us != 0);
        return true;
    }
};

// Where the projected work ends: a frame counted from the planned one and the
// estimate already placed in it (Cursor, schedule.rs:321).
struct Cursor {
    uint64_t frame = 0, spent = 0;
    uint64_t instant(const bl_frame_info& planned) const {
        return sat_add(sat_add(planned.start_us, sat_mul(frame, planned.period_us)), spent);
    }
};

struct Budgets {
    uint64_t now, later;
    uint64_t of(uint64_t frame) const { return frame == 0 ? now : later; }

    // lays `slices` in order onto frames from `from` (Budgets::place,
    // schedule.rs:373): `ok` false when a slice fits no empty later frame;
    // `count_now` = leading slices that landed in the planned frame
    bool place(Cursor from, const uint32_t* slices, size_t n, const bl_cost* cost, Cursor* end,
               size_t* count_now) const {
        Cursor at = from;
        size_t now = 0;
        for (size_t k = 0; k < n; ++k) {
            const uint64_t est = bl_cost_planning_estimate(cost, slices[k]);
            for (;;) {
                const uint64_t after = sat_add(at.spent, est);
                if (after <= of(at.frame)) {
                    at.spent = after;
                    break;
                }
                if (at.frame > 0 && at.spent == 0) {
                    *count_now = now;
                    return false;
                }
                at = Cursor{sat_add(at.frame, 1), 0};
            }
            if (at.frame == 0) ++now;
        }
        *end = at;
        *count_now = now;
        return true;
    }
};

enum class Fate { Passed, Abandoned, Late, Kept };

struct Job {
    uint64_t id, input;
    std::vector<uint32_t> slices;
    size_t scheduled = 0;
    Due deadline;
    bool abandoned = false;

    bool complete() const { return scheduled >= slices.size(); }
    bool passed(const bl_frame_info& f) const {
        uint64_t l;
        return !deadline.frames_left(f, &l);
    }
    // Job::fate (schedule.rs:452)
    Fate fate(Cursor from, const bl_frame_info& f, Budgets b, const bl_cost* cost, bool behind,
              size_t* now, Cursor* end) const {
        uint64_t left = 0;
        *now = 0;
        if (!deadline.frames_left(f, &left)) return Fate::Passed;
        if (complete()) {
            *end = from;
            return Fate::Kept;
        }
        Cursor e;
        size_t cnt = 0;
        const bool ok = b.place(from, slices.data() + scheduled, slices.size() - scheduled, cost, &e,
                                &cnt);
        if (ok && e.frame <= left) {
            *now = cnt, *end = e;
            return Fate::Kept;
        }
        if (behind) return Fate::Abandoned;
        *now = cnt;
        return Fate::Late;
    }
};

}  // namespace sched
}  // namespace bl

struct bl_scheduler {
    bl_sync_policy policy{};
    int32_t miss = BL_MISS_HOLD_PREVIOUS;
    uint64_t expected = 0;
    uint64_t next_job = 0;
    uint64_t margin = 0;
    bl::sched::BeatMap beats;
    std::vector<bl::sched::Job> pending;
    // the last plan
    std::vector<bl_slice_run> runs;
    std::vector<bl_delivery> delivered;
    std::vector<bl_missed> missed;

    bool on_beat() const { return policy.kind == BL_SYNC_ON_BEAT; }

    // where the work of the jobs kept ahead of a job being submitted ends
    // (projected_end, schedule.rs:680): every pending job has one behind it
    bl::sched::Cursor projected_end(const bl_frame_info& f, bl::sched::Budgets b,
                                    const bl_cost* cost) const {
        bl::sched::Cursor at;
        for (const auto& job : pending) {
            size_t now = 0;
            bl::sched::Cursor end;
            if (job.fate(at, f, b, cost, true, &now, &end) == bl::sched::Fate::Kept) at = end;
        }
        return at;
    }
};

namespace {

bl_due to_c(const bl::sched::Due& d) {
    bl_due o{};
    o.kind = d.beat ? BL_DUE_BEAT : BL_DUE_FRAME;
    o.at = d.at;
    return o;
}

}  // namespace

extern "C" {

uint64_t bl_budget_for_frame(uint64_t period_us, uint64_t render_us, uint64_t margin_us) {
    return bl::sched::sat_sub(bl::sched::sat_sub(period_us, render_us), margin_us);
}

int bl_beat_map_next(const uint64_t* grids, size_t n, uint64_t t, uint64_t* out) {
    if (grids == nullptr || n == 0 || out == nullptr)
        return bl::fail(BL_ERR_INVALID, "beat map: no grid");
    bl::sched::BeatMap m;
    for (size_t i = 0; i < n; ++i) {
        if (grids[3 * i + 2] == 0) return bl::fail(BL_ERR_INVALID, "beat length must be greater than zero");
        if (i == 0) m.grids.push_back({0, grids[1], grids[2]});
        else m.replace_from(grids[3 * i], grids[3 * i + 1], grids[3 * i + 2]);
    }
    *out = m.next(t);
    return BL_OK;
}

int bl_scheduler_create(const bl_sync_policy* policy, int32_t miss, uint64_t expected_budget_us,
                        bl_scheduler** out) {
    if (policy == nullptr || out == nullptr) return bl::fail(BL_ERR_INVALID, "scheduler: null argument");
    *out = nullptr;
    if (policy->kind < BL_SYNC_FIXED_LATENCY || policy->kind > BL_SYNC_ON_BEAT)
        return bl::fail(BL_ERR_INVALID, "scheduler: sync policy %d", policy->kind);
    if (miss != BL_MISS_HOLD_PREVIOUS && miss != BL_MISS_DROP)
        return bl::fail(BL_ERR_INVALID, "scheduler: miss policy %d", miss);
    if (policy->kind == BL_SYNC_ON_BEAT && policy->grid_beat_us == 0)
        return bl::fail(BL_ERR_INVALID, "beat length must be greater than zero (ZeroBeat)");
    bl_scheduler* s = new bl_scheduler();
    s->policy = *policy;
    s->miss = miss;
    s->expected = expected_budget_us;
    if (s->on_beat()) {
        s->margin = policy->margin_us;
        s->beats.grids.push_back({0, policy->grid_origin_us, policy->grid_beat_us});
    }
    *out = s;
    return BL_OK;
}

void bl_scheduler_destroy(bl_scheduler* s) { delete s; }

void bl_scheduler_set_expected_budget(bl_scheduler* s, uint64_t expected_us) {
    if (s) s->expected = expected_us;
}

uint64_t bl_scheduler_expected_budget(const bl_scheduler* s) { return s ? s->expected : 0; }

int bl_scheduler_replace_beat_grid(bl_scheduler* s, uint64_t from_us, uint64_t origin_us,
                                   uint64_t beat_us) {
    if (s == nullptr) return bl::fail(BL_ERR_INVALID, "scheduler: null");
    if (!s->on_beat()) return bl::fail(BL_ERR_INVALID, "only an OnBeat scheduler has a beat grid (NotOnBeat)");
    if (beat_us == 0) return bl::fail(BL_ERR_INVALID, "beat length must be greater than zero (ZeroBeat)");
    s->beats.replace_from(from_us, origin_us, beat_us);
    return BL_OK;
}

int bl_scheduler_submit(bl_scheduler* s, const bl_frame_info* input, const uint32_t* slices,
                        size_t n, const bl_cost* cost, uint64_t* job) {
    using namespace bl::sched;
    if (s == nullptr || input == nullptr || cost == nullptr)
        return bl::fail(BL_ERR_INVALID, "scheduler: null argument");
    if (n == 0 || slices == nullptr) return bl::fail(BL_ERR_INVALID, "a job needs at least one slice (EmptyJob)");
    Due d{};
    if (!s->on_beat()) {
        const uint32_t frames = s->policy.kind == BL_SYNC_SAME_FRAME ? 0 : s->policy.frames;
        d = Due{false, sat_add(input->index, frames)};
    } else {
        const Budgets b{s->expected, s->expected};
        const Cursor ahead = s->projected_end(*input, b, cost);
        Cursor end;
        size_t now = 0;
        uint64_t finish;
        if (b.place(ahead, slices, n, cost, &end, &now)) {
            finish = end.instant(*input);
        } else {
            finish = input->start_us;
            for (size_t k = 0; k < n; ++k) finish = sat_add(finish, bl_cost_planning_estimate(cost, slices[k]));
        }
        d = Due{true, s->beats.next(sat_add(finish, s->margin))};
    }
    Job j;
    j.id = s->next_job;
    j.input = input->index;
    j.slices.assign(slices, slices + n);
    j.deadline = d;
    s->next_job = sat_add(s->next_job, 1);
    s->pending.push_back(std::move(j));
    if (job) *job = s->pending.back().id;
    return BL_OK;
}

int bl_scheduler_plan_frame(bl_scheduler* s, const bl_frame_info* frame, uint64_t budget_us,
                            const bl_cost* cost, bl_frame_plan_info* info) {
    using namespace bl::sched;
    if (s == nullptr || frame == nullptr || cost == nullptr)
        return bl::fail(BL_ERR_INVALID, "scheduler: null argument");
    if (s->on_beat()) s->beats.forget_before(frame->start_us);
    const Budgets b{budget_us, s->expected};
    s->runs.clear();
    s->delivered.clear();
    s->missed.clear();
    uint64_t spent = 0;
    Cursor at;
    // the last job this plan does not report missed for a passed deadline
    long last_waiting = -1;
    for (size_t i = 0; i < s->pending.size(); ++i)
        if (!s->pending[i].passed(*frame)) last_waiting = static_cast<long>(i);
    auto hand_out = [&](Job& job, size_t count) {
        for (size_t c = 0; c < count && job.scheduled < job.slices.size(); ++c) {
            bl_slice_run r{};
            r.job = job.id;
            r.slice = job.slices[job.scheduled];
            r.position = job.scheduled;
            s->runs.push_back(r);
            spent = sat_add(spent, bl_cost_planning_estimate(cost, r.slice));
            job.scheduled += 1;
        }
    };
    for (size_t i = 0; i < s->pending.size(); ++i) {
        Job& job = s->pending[i];
        const bool behind = last_waiting >= 0 && static_cast<long>(i) < last_waiting;
        size_t now = 0;
        Cursor end;
        switch (job.fate(at, *frame, b, cost, behind, &now, &end)) {
            case Fate::Passed: break;
            case Fate::Abandoned: job.abandoned = true; break;
            case Fate::Late: hand_out(job, now); break;
            case Fate::Kept:
                hand_out(job, now);
                at = end;
                break;
        }
    }
    std::vector<Job> keep;
    for (Job& job : s->pending) {
        if (!(job.abandoned || job.deadline.reached(*frame))) {
            keep.push_back(std::move(job));
            continue;
        }
        if (!job.abandoned && job.complete() && job.deadline.on_time(*frame)) {
            s->delivered.push_back(bl_delivery{job.id, job.input});
        } else {
            bl_missed m{};
            m.job = job.id;
            m.input = job.input;
            m.due = to_c(job.deadline);
            m.policy = s->miss;
            s->missed.push_back(m);
        }
    }
    s->pending.swap(keep);
    if (info) {
        info->runs = s->runs.size();
        info->delivered = s->delivered.size();
        info->missed = s->missed.size();
        info->spent_estimate_us = spent;
        info->budget_us = budget_us;
    }
    return BL_OK;
}

size_t bl_scheduler_plan_runs(const bl_scheduler* s, bl_slice_run* out, size_t cap) {
    if (s == nullptr) return 0;
    const size_t n = std::min(cap, s->runs.size());
    if (out) std::copy(s->runs.begin(), s->runs.begin() + n, out);
    return s->runs.size();
}

size_t bl_scheduler_plan_delivered(const bl_scheduler* s, bl_delivery* out, size_t cap) {
    if (s == nullptr) return 0;
    const size_t n = std::min(cap, s->delivered.size());
    if (out) std::copy(s->delivered.begin(), s->delivered.begin() + n, out);
    return s->delivered.size();
}

size_t bl_scheduler_plan_missed(const bl_scheduler* s, bl_missed* out, size_t cap) {
    if (s == nullptr) return 0;
    const size_t n = std::min(cap, s->missed.size());
    if (out) std::copy(s->missed.begin(), s->missed.begin() + n, out);
    return s->missed.size();
}

size_t bl_scheduler_pending(const bl_scheduler* s) { return s ? s->pending.size() : 0; }

int bl_scheduler_due(const bl_scheduler* s, uint64_t job, bl_due* out) {
    if (s == nullptr) return 0;
    for (const auto& j : s->pending)
        if (j.id == job) {
            if (out) *out = to_c(j.deadline);
            return 1;
        }
    return 0;
}

}  // extern "C"
