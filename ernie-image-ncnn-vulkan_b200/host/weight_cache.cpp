// Weight placement and the per-request weight cache of the C++ host surface (include/ernie_b200/ernie.h).
//
// Both are small policies whose observable behaviour is fixed by the reference's contract tests
// (tests/test_weight_placement.cpp:38-78, tests/test_weight_session.cpp:36-131): which requests go to
// host memory and why, which prepared blocks stay cached across a repeated 36-block scan, when idle
// entries are dropped under RAM pressure, and what each counter reports. On a B200 every block stays
// resident in HBM, so these run only for callers that mirror the reference's streaming setup.
#include "ernie_b200/ernie.h"
#include <algorithm>
#include <array>
#include <stdexcept>
#include <utility>

namespace ernie
{
WeightMemory parse_weight_memory(const std::string &value)
{
    static const std::pair<const char *, WeightMemory> names[] = {
        {"auto", WeightMemory::Auto}, {"device", WeightMemory::Device}, {"host", WeightMemory::Host}};
    for (const auto &[name, mode] : names)
        if (value == name) return mode;
    throw std::invalid_argument("DiT weights must be auto, device, or host");
}

namespace
{
// Device bytes still free under the budget (zero when usage already exceeds it).
std::uint64_t unused_budget(const DeviceMemoryBudget &m) { return m.budget_bytes > m.usage_bytes ? m.budget_bytes - m.usage_bytes : 0; }

// True when `weight` bytes fit in `available` after keeping `reserve` bytes back. A sum that does not
// fit in 64 bits cannot fit in any budget.
bool fits_after_reserve(std::uint64_t available, std::uint64_t reserve, std::uint64_t weight)
{
    std::uint64_t needed = 0;
    if (__builtin_add_overflow(reserve, weight, &needed)) return false;
    return needed <= available;
}

WeightPlacementDecision decided(WeightPlacementDecision d, bool host, const char *reason)
{
    d.host = host;
    d.reason = reason;
    return d;
}
} // namespace

// Precedence: an explicit mode, then the shape's preference for host memory, then the device budget;
// with no budget reading the weights go to the device and the reason says "unavailable".
WeightPlacementDecision choose_weight_placement(WeightMemory mode, bool shape_prefers_host, std::uint64_t weight_bytes,
                                                std::uint64_t reserve_bytes, std::optional<DeviceMemoryBudget> memory)
{
    WeightPlacementDecision d;
    d.weight_bytes = weight_bytes;
    d.reserve_bytes = reserve_bytes;
    if (memory) d.available_bytes = unused_budget(*memory);
    switch (mode)
    {
    case WeightMemory::Host: return decided(d, true, "explicit");
    case WeightMemory::Device: return decided(d, false, "explicit");
    case WeightMemory::Auto: break;
    }
    if (shape_prefers_host) return decided(d, true, "shape");
    if (!d.available_bytes) return d;
    const bool fits = fits_after_reserve(*d.available_bytes, reserve_bytes, weight_bytes);
    return decided(d, !fits, fits ? "available" : "budget");
}

WeightPlacement::WeightPlacement(WeightMemory mode, std::uint64_t reserve_bytes, BudgetReader reader, Observer observer)
    : mode_(mode), reserve_bytes_(reserve_bytes), reader_(std::move(reader)), observer_(std::move(observer))
{
}

bool WeightPlacement::use_host(const std::string &component, std::uint64_t weight_bytes, bool shape_prefers_host,
                               bool cache_prefers_host, const char *host_reason)
{
    // Only the automatic mode reads the budget, once per request, so a changing budget is seen.
    const bool automatic = mode_ == WeightMemory::Auto;
    std::optional<DeviceMemoryBudget> memory;
    if (automatic)
    {
        if (reader_) memory = reader_();
        if (!memory) ++unavailable_queries_;
    }
    WeightPlacementDecision d = choose_weight_placement(mode_, shape_prefers_host, weight_bytes, reserve_bytes_, memory);
    if (automatic && cache_prefers_host) d = decided(d, true, host_reason);
    ++(d.host ? host_requests_ : device_requests_);
    if (observer_) observer_(component, d);
    return d.host;
}

WeightPlacement::BudgetReader cuda_memory_budget_reader(GpuContext &ctx)
{
    ernie_cuda_context *handle = ctx.handle();
    return [handle]() -> std::optional<DeviceMemoryBudget> {
        uint64_t free_bytes = 0, total = 0;
        if (ernie_cuda_context_memory(handle, &free_bytes, &total) != ERNIE_CUDA_OK) return std::nullopt;
        return DeviceMemoryBudget{total, total - free_bytes};
    };
}

// ---- WeightSession ----------------------------------------------------------------------------------
//
// Slots are indexed by block (a DiT has at most 36). A block's payload is either idle in its slot, out
// on the one lease, or not cached. The cache admits blocks while their measured size fits the host
// budget and RAM above the reserve allows, and never replaces an admitted block with a later one: in
// a repeated scan of the same blocks the admitted prefix keeps hitting while the rest stream, where
// least-recently-used replacement would miss every block. Under RAM pressure idle slots are dropped
// from the highest block index down, so the prefix is the last to go.
namespace
{
constexpr std::size_t kBlockSlots = 36;
}

struct WeightSession::State
{
    struct Idle
    {
        Payload payload;
        std::uint64_t charge = 0;
    };
    WeightBudget budget;
    AvailableReader ram;
    Inspector measure;
    WeightSessionStats stats;
    std::array<std::optional<Idle>, kBlockSlots> slots;
    std::array<std::string, kBlockSlots> bound; // the identity each block was first acquired with
    const void *request = nullptr;              // the request the session serves (first acquire binds it)
    bool leased = false, closed = false;

    // Host RAM above the reserve, or nothing when it cannot be read (counted) or is below the reserve.
    std::optional<std::uint64_t> ram_above_reserve()
    {
        const std::optional<std::uint64_t> available = ram ? ram() : std::nullopt;
        if (!available)
        {
            ++stats.unavailable_queries;
            return std::nullopt;
        }
        if (*available < budget.reserve_bytes) return std::nullopt;
        return *available - budget.reserve_bytes;
    }
    bool ram_allows(std::uint64_t bytes)
    {
        const auto spare = ram_above_reserve();
        return spare && *spare >= bytes;
    }
    std::uint64_t budget_left() const { return budget.host_bytes - stats.live_bytes; }
    void uncharge(std::uint64_t charge)
    {
        if (!charge) return;
        stats.live_bytes -= charge;
        --stats.cached_nets;
    }
    void evict(std::size_t block)
    {
        uncharge(slots[block]->charge);
        slots[block].reset();
        ++stats.evictions;
    }
    // Drops idle slots, highest block first, until `block` (cached or about to be loaded at
    // `estimate` bytes) has RAM headroom or nothing idle is left.
    void relieve_pressure(std::size_t block, std::uint64_t estimate)
    {
        for (std::size_t b = kBlockSlots; b-- > 0;)
        {
            if (!slots[b]) continue;
            if (ram_allows(slots[block] ? 0 : estimate)) return;
            evict(b);
        }
    }
    // Charges a freshly loaded payload to the cache if its measured size fits; returns the charge.
    std::uint64_t admit(const Payload &payload)
    {
        const std::optional<std::uint64_t> size = measure(payload);
        if (!size || *size == 0 || *size > budget_left() || !ram_allows(0)) return 0;
        stats.live_bytes += *size;
        stats.peak_bytes = std::max(stats.peak_bytes, stats.live_bytes);
        ++stats.cached_nets;
        stats.peak_nets = std::max(stats.peak_nets, stats.cached_nets);
        ++stats.admissions;
        return *size;
    }
    // A lease comes back: a completed, charged payload returns to its slot unless the session was
    // cancelled; anything else is discarded and its charge released.
    void settle(std::size_t block, Payload payload, std::uint64_t charge, bool completed)
    {
        leased = false;
        if (completed && charge && !closed)
        {
            slots[block] = Idle{std::move(payload), charge};
            return;
        }
        payload.reset();
        uncharge(charge);
    }
};

WeightSession::WeightSession(WeightBudget budget, AvailableReader available, Inspector inspect)
    : state_(std::make_shared<State>())
{
    state_->budget = budget;
    state_->ram = std::move(available);
    state_->measure = std::move(inspect);
}

WeightSession::~WeightSession() { cancel(); }
WeightSessionStats WeightSession::stats() const { return state_->stats; }
bool WeightSession::contains(std::size_t block) const { return block < kBlockSlots && state_->slots[block].has_value(); }

void WeightSession::cancel()
{
    State &s = *state_;
    s.closed = true;
    for (std::size_t b = kBlockSlots; b-- > 0;)
        if (s.slots[b]) s.evict(b);
}

WeightSession::Lease WeightSession::acquire(std::size_t block, const std::string &identity, const void *request,
                                            std::uint64_t estimate, const Loader &loader)
{
    State &s = *state_;
    if (s.closed) throw std::logic_error("Weight session is cancelled");
    if (s.leased) throw std::logic_error("Weight session lease is still outstanding");
    if (block >= kBlockSlots || !request || !loader || identity.empty())
        throw std::invalid_argument("Invalid weight session request");
    if (s.request && s.request != request) throw std::logic_error("Weight session belongs to another request");
    s.request = request;
    std::string &bound = s.bound[block];
    if (!bound.empty() && bound != identity) throw std::logic_error("Weight session block changed model identity");
    bound = identity;

    if (s.budget.host_bytes) s.relieve_pressure(block, estimate);
    if (std::optional<State::Idle> &slot = s.slots[block])
    {
        State::Idle hit = std::move(*slot);
        slot.reset();
        ++s.stats.hits;
        s.leased = true;
        return Lease(state_, block, std::move(hit.payload), hit.charge);
    }
    const bool cacheable = s.measure && s.budget.host_bytes && estimate <= s.budget_left() && s.ram_allows(estimate);
    Payload payload = loader(cacheable); // a throwing loader leaves the session as it was
    if (!payload) throw std::runtime_error("Weight loader returned no payload");
    ++s.stats.loads;
    const std::uint64_t charge = cacheable ? s.admit(payload) : 0;
    s.leased = true;
    return Lease(state_, block, std::move(payload), charge);
}

WeightSession::Lease::Lease(std::shared_ptr<State> state, std::size_t block, Payload payload, std::uint64_t charge)
    : state_(std::move(state)), block_(block), payload_(std::move(payload)), charge_(charge)
{
}

WeightSession::Lease::Lease(Lease &&other) noexcept
    : state_(std::exchange(other.state_, nullptr)), block_(other.block_), payload_(std::move(other.payload_)),
      charge_(std::exchange(other.charge_, 0))
{
}

WeightSession::Lease &WeightSession::Lease::operator=(Lease &&other) noexcept
{
    if (this == &other) return *this;
    release(false);
    state_ = std::exchange(other.state_, nullptr);
    block_ = other.block_;
    payload_ = std::move(other.payload_);
    charge_ = std::exchange(other.charge_, 0);
    return *this;
}

WeightSession::Lease::~Lease() { release(false); }

const WeightSession::Payload &WeightSession::Lease::payload() const
{
    if (!payload_) throw std::logic_error("Weight lease no longer holds a payload");
    return payload_;
}

void WeightSession::Lease::complete()
{
    if (!payload_) throw std::logic_error("Weight lease no longer holds a payload");
    release(true);
}

void WeightSession::Lease::release(bool completed)
{
    const std::shared_ptr<State> state = std::exchange(state_, nullptr);
    if (state && payload_) state->settle(block_, std::move(payload_), charge_, completed);
}
} // namespace ernie
