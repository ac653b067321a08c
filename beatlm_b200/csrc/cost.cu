// Measured slice costs for the frame scheduler: the reference's CostModel
// (crates/beatlm-core/src/cost.rs:726-966) with its four estimators, fed here
// from the cudaEvent slice timer instead of wgpu timestamp queries. Host code
// only; the scheduler plans with these numbers, so the statistics, their
// rounding and their error cases follow the reference exactly (a plan made
// from the same measurements must be the same plan).
#include <algorithm>
#include <cmath>
#include <map>
#include <vector>

#include "host.h"

namespace bl {
namespace cost {

constexpr size_t kMaxWindow = 4096;   // MAX_WINDOW, cost.rs:294
constexpr uint32_t kWarmSamples = 5;  // WARM_SAMPLES, cost.rs:671

uint32_t sat_inc(uint32_t v) { return v == UINT32_MAX ? v : v + 1; }
uint64_t sat_inc(uint64_t v) { return v == UINT64_MAX ? v : v + 1; }

// Rounds up to whole microseconds; NaN and negatives are zero, 2^64 and above
// saturate (f64_to_micros_ceil, cost.rs:1001).
uint64_t ceil_micros(double v) {
    v = std::ceil(std::fmax(v, 0.0));
    return v >= 18446744073709551616.0 ? UINT64_MAX : static_cast<uint64_t>(v);
}

// 1-based nearest rank of q among n values; a product within 1e-9 of a whole
// number is that number, so 0.55 of 100 is rank 55 (nearest_rank, cost.rs:653).
size_t nearest_rank(double q, size_t n) {
    const double product = q * static_cast<double>(n);
    const double whole = std::round(product);
    const double r = std::fabs(product - whole) < 1e-9 ? whole : std::ceil(product);
    const size_t rank = r > 0.0 ? static_cast<size_t>(r) : 0;
    return std::min(std::max(rank, size_t(1)), std::max(n, size_t(1)));
}

// median x scale rounded up, a product within a billionth of a whole number
// being that number (scaled_ceil, cost.rs:988)
uint64_t scaled_ceil(uint64_t median, double scale) {
    const double product = static_cast<double>(median) * scale;
    const double whole = std::round(product);
    return ceil_micros(std::fabs(product - whole) <= std::fabs(product) * 1e-9 ? whole : product);
}

// Exponentially weighted mean and variance (Ewma, cost.rs:486-526).
struct Ewma {
    double mean = 0.0, var = 0.0;
    uint32_t samples = 0;
    void first(double x) { mean = x, var = 0.0, samples = 1; }
    void fold(double x, double alpha) {
        const double diff = x - mean;
        const double incr = alpha * diff;
        mean += incr;
        var = (1.0 - alpha) * (var + diff * incr);
        samples = sat_inc(samples);
    }
    double stddev() const { return std::sqrt(std::fmax(var, 0.0)); }
};

// The last `capacity` measurements and one or two nearest-rank reads of them
// (Window, cost.rs:528-596): the read is a selection, not a sort.
struct Window {
    std::vector<uint64_t> ring, scratch;
    size_t next = 0;
    uint64_t estimate = 0, second = 0;
    uint32_t samples = 0;

    uint64_t select(double q) {
        const size_t k = nearest_rank(q, scratch.size()) - 1;
        std::nth_element(scratch.begin(), scratch.begin() + k, scratch.end());
        return scratch[k];
    }
    void fold(uint64_t x, size_t capacity, double q, const double* q2) {
        if (ring.size() < capacity) ring.push_back(x);
        else ring[next] = x;
        next = (next + 1) % capacity;
        samples = sat_inc(samples);
        scratch.assign(ring.begin(), ring.end());
        estimate = select(q);
        second = q2 != nullptr ? select(*q2) : estimate;
    }
};

struct Ratio {
    double ratio, weight;
};

// The first ratio (ascending) at which the cumulative weight reaches q of the
// total, less a billionth of it (weighted_rank, cost.rs:636).
double weighted_rank(const std::vector<Ratio>& sorted, double q) {
    double total = 0.0;
    for (const Ratio& r : sorted) total += r.weight;
    const double target = std::fma(q, total, -(total * 1e-9));
    double reached = 0.0;
    for (const Ratio& r : sorted) {
        reached += r.weight;
        if (reached >= target) return r.ratio;
    }
    return sorted.empty() ? 1.0 : sorted.back().ratio;
}

// The last frames' measured-over-planned ratios (Frames, cost.rs:589-630).
struct Frames {
    std::vector<Ratio> ring, scratch;
    size_t next = 0;
    double scale = 1.0;
    uint64_t recorded = 0;

    void fold(Ratio f, size_t capacity, double q) {
        if (ring.size() < capacity) ring.push_back(f);
        else ring[next] = f;
        next = (next + 1) % capacity;
        recorded = sat_inc(recorded);
        if (ring.size() < capacity) return;  // read only from a full window
        scratch = ring;
        std::sort(scratch.begin(), scratch.end(),
                  [](const Ratio& a, const Ratio& b) { return a.ratio < b.ratio; });
        const double s = weighted_rank(scratch, q);
        scale = std::isnan(s) ? 1.0 : std::fmax(s, 1.0);
    }
};

struct State {
    Ewma ewma;
    Window all;     // WindowedQuantile: the window; FrameScaled: every measurement
    Window looped;  // FrameScaled: the loop's measurements alone
    bool warm() const { return looped.samples >= kWarmSamples; }
};

const char* error_text(int code) {
    switch (code) {
        case BL_COST_INVALID_ALPHA: return "alpha must be finite and in (0, 1]";
        case BL_COST_INVALID_SIGMAS: return "sigmas must be finite and non-negative";
        case BL_COST_INVALID_WINDOW: return "window must be in 1..=MAX_WINDOW";
        case BL_COST_INVALID_QUANTILE: return "quantile must be finite and in [0, 1]";
        case BL_COST_INVALID_FRAME_WINDOW: return "frame window must be in 1..=MAX_WINDOW";
        case BL_COST_INVALID_CAP: return "cap must be finite and non-negative";
        default: return "unknown estimator";
    }
}

// Estimator::validate (cost.rs:427-480): the first parameter out of range.
int validate(const bl_estimator& e) {
    auto unit = [](double x) { return std::isfinite(x) && x > 0.0 && x <= 1.0; };
    auto non_negative = [](double x) { return std::isfinite(x) && x >= 0.0; };
    auto rank = [](double q) { return std::isfinite(q) && q >= 0.0 && q <= 1.0; };
    auto window = [](uint32_t w) { return w >= 1 && w <= kMaxWindow; };
    switch (e.kind) {
        case BL_EST_MEAN_PLUS_SIGMAS:
            if (!unit(e.alpha)) return BL_COST_INVALID_ALPHA;
            if (!non_negative(e.sigmas)) return BL_COST_INVALID_SIGMAS;
            return 0;
        case BL_EST_WINDOWED_QUANTILE:
            if (!window(e.window)) return BL_COST_INVALID_WINDOW;
            if (!rank(e.quantile)) return BL_COST_INVALID_QUANTILE;
            return 0;
        case BL_EST_FRAME_SCALED:
            if (!window(e.window)) return BL_COST_INVALID_WINDOW;
            if (!window(e.frame_window)) return BL_COST_INVALID_FRAME_WINDOW;
            if (!rank(e.quantile)) return BL_COST_INVALID_QUANTILE;
            return 0;
        case BL_EST_CAPPED_DEVIATION:
            if (!unit(e.alpha)) return BL_COST_INVALID_ALPHA;
            if (!non_negative(e.sigmas)) return BL_COST_INVALID_SIGMAS;
            if (!non_negative(e.cap)) return BL_COST_INVALID_CAP;
            return 0;
        default:
            return BL_COST_UNKNOWN_ESTIMATOR;
    }
}

}  // namespace cost
}  // namespace bl

struct bl_cost {
    uint64_t prior = 0;
    bl_estimator est{};
    std::map<uint32_t, bl::cost::State> stats;  // ordered: same input, same output
    bl::cost::Frames frames;                      // FrameScaled only

    bool scaled() const { return est.kind == BL_EST_FRAME_SCALED; }
    const bl::cost::State* find(uint32_t slice) const {
        auto it = stats.find(slice);
        return it == stats.end() ? nullptr : &it->second;
    }

    void fold(uint32_t slice, uint64_t measured, bool in_loop) {
        auto it = stats.find(slice);
        const bool fresh = it == stats.end();
        bl::cost::State& s = fresh ? stats[slice] : it->second;
        switch (est.kind) {
            case BL_EST_MEAN_PLUS_SIGMAS:
            case BL_EST_CAPPED_DEVIATION:
                if (fresh) s.ewma.first(static_cast<double>(measured));
                else s.ewma.fold(static_cast<double>(measured), est.alpha);
                break;
            case BL_EST_WINDOWED_QUANTILE:
                s.all.fold(measured, est.window, est.quantile, nullptr);
                break;
            case BL_EST_FRAME_SCALED: {
                const double median = 0.5;
                s.all.fold(measured, est.window, est.quantile, &median);
                if (in_loop) s.looped.fold(measured, est.window, 0.5, nullptr);
                break;
            }
        }
    }

    uint64_t estimate(uint32_t slice) const {
        const bl::cost::State* s = find(slice);
        if (s == nullptr) return prior;
        switch (est.kind) {
            case BL_EST_MEAN_PLUS_SIGMAS:
                return bl::cost::ceil_micros(std::fma(est.sigmas, s->ewma.stddev(), s->ewma.mean));
            case BL_EST_CAPPED_DEVIATION: {
                const double pad = std::fmin(est.sigmas * s->ewma.stddev(),
                                             est.cap * std::fmax(s->ewma.mean, 0.0));
                return bl::cost::ceil_micros(s->ewma.mean + pad);
            }
            case BL_EST_WINDOWED_QUANTILE:
                return s->all.estimate;
            default:  // FrameScaled: the loop median once warm, else the median of all
                return s->warm() ? s->looped.estimate : s->all.second;
        }
    }

    int32_t frame_scale(double* scale, uint64_t* recorded, uint64_t* needed) const {
        if (!scaled()) return BL_FRAME_SCALE_NONE;
        if (frames.ring.size() < est.frame_window) {
            if (recorded) *recorded = frames.ring.size();
            if (needed) *needed = est.frame_window;
            return BL_FRAME_SCALE_WARMING_UP;
        }
        if (scale) *scale = frames.scale;
        return BL_FRAME_SCALE_MEASURED;
    }
};

extern "C" {

void bl_estimator_default(bl_estimator* out) {
    if (out == nullptr) return;
    *out = bl_estimator{};
    out->kind = BL_EST_WINDOWED_QUANTILE;  // Estimator::default, cost.rs:416-425
    out->window = 32;
    out->quantile = 0.9;
}

int bl_cost_create(uint64_t prior_us, const bl_estimator* est, bl_cost** out, int32_t* cost_error) {
    if (cost_error) *cost_error = 0;
    if (est == nullptr || out == nullptr) return bl::fail(BL_ERR_INVALID, "cost: null argument");
    *out = nullptr;
    const int e = bl::cost::validate(*est);
    if (e != 0) {
        if (cost_error) *cost_error = e;
        return bl::fail(BL_ERR_INVALID, "cost: %s", bl::cost::error_text(e));
    }
    bl_cost* c = new bl_cost();
    c->prior = prior_us;
    c->est = *est;
    *out = c;
    return BL_OK;
}

int bl_cost_clone(const bl_cost* c, bl_cost** out) {
    if (c == nullptr || out == nullptr) return bl::fail(BL_ERR_INVALID, "cost: null argument");
    *out = new bl_cost(*c);
    return BL_OK;
}

void bl_cost_destroy(bl_cost* c) { delete c; }

int bl_cost_estimator(const bl_cost* c, bl_estimator* out) {
    if (c == nullptr || out == nullptr) return bl::fail(BL_ERR_INVALID, "cost: null argument");
    *out = c->est;
    return BL_OK;
}

void bl_cost_record(bl_cost* c, uint32_t slice, uint64_t measured_us) {
    if (c) c->fold(slice, measured_us, true);
}

void bl_cost_record_calibration(bl_cost* c, uint32_t slice, uint64_t measured_us) {
    if (c) c->fold(slice, measured_us, false);
}

int bl_cost_frame_estimate(const bl_cost* c, uint32_t slice, uint64_t* out) {
    if (c == nullptr) return 0;
    const bl::cost::State* s = c->find(slice);
    if (c->scaled()) {  // warm slices only (cost.rs:851-860)
        if (s == nullptr || !s->warm()) return 0;
        if (out) *out = s->looped.estimate;
        return 1;
    }
    if (out) *out = c->estimate(slice);
    return 1;
}

void bl_cost_record_frame(bl_cost* c, uint64_t predicted_us, uint64_t measured_us) {
    if (c == nullptr || !c->scaled() || predicted_us == 0) return;
    const double w = static_cast<double>(predicted_us);
    c->frames.fold({static_cast<double>(measured_us) / w, w}, c->est.frame_window, c->est.quantile);
}

int32_t bl_cost_frame_scale(const bl_cost* c, double* scale, uint64_t* recorded, uint64_t* needed) {
    return c ? c->frame_scale(scale, recorded, needed) : BL_FRAME_SCALE_NONE;
}

uint64_t bl_cost_frames_recorded(const bl_cost* c) {
    return c && c->scaled() ? c->frames.recorded : 0;
}

uint64_t bl_cost_planning_estimate(const bl_cost* c, uint32_t slice) {
    if (c == nullptr) return 0;
    const bl::cost::State* s = c->find(slice);
    if (c->scaled() && s != nullptr) {
        double scale = 1.0;
        if (c->frame_scale(&scale, nullptr, nullptr) == BL_FRAME_SCALE_MEASURED && s->warm())
            return bl::cost::scaled_ceil(s->looped.estimate, scale);
        return s->all.estimate;  // the frame quantile of every measurement
    }
    return c->estimate(slice);
}

uint64_t bl_cost_estimate(const bl_cost* c, uint32_t slice) { return c ? c->estimate(slice) : 0; }

uint32_t bl_cost_samples(const bl_cost* c, uint32_t slice) {
    if (c == nullptr) return 0;
    const bl::cost::State* s = c->find(slice);
    if (s == nullptr) return 0;
    switch (c->est.kind) {
        case BL_EST_MEAN_PLUS_SIGMAS:
        case BL_EST_CAPPED_DEVIATION:
            return s->ewma.samples;
        default:
            return s->all.samples;
    }
}

uint64_t bl_micros_nearest(double micros) {
    // a timer duration in whole microseconds, rounded to nearest (the
    // reference's ticks_to_micros, crates/beatlm/src/gpu/timer.rs:781-800)
    const double r = std::round(micros);
    if (!(r > 0.0)) return 0;
    return r >= 18446744073709551616.0 ? UINT64_MAX : static_cast<uint64_t>(r);
}

size_t bl_cost_record_passes(bl_cost* c, const bl_slice_time* passes, size_t n, int calibration) {
    if (c == nullptr || passes == nullptr) return 0;
    for (size_t i = 0; i < n; ++i)
        c->fold(passes[i].kernel, bl_micros_nearest(passes[i].micros), calibration == 0);
    return n;
}

}  // extern "C"
