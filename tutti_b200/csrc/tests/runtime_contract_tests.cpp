// Contract suite of StorageRuntime over the mock DataPath kit: the behaviours
// a DataPath author and a runtime user rely on (partial acceptance, handle
// hygiene, budgets, lifecycle, concurrency), one case per rule.
// Parity: the rules of reference
// tests/storage_runtime/contract/storage_runtime_contract_test.cpp; the cases
// are written against this runtime's API.

#include <atomic>
#include <thread>

#include "harness.h"

using namespace tutti;
using namespace tutti::native_tests;

namespace {
HostSubmitContext host_ctx() { return HostSubmitContext{ExecutionDomain::HOST_EXECUTION, -1, nullptr}; }

bool completed(StorageRuntime& rt, const IoHandle& h, std::uint64_t bytes) {
    auto w = rt.wait(h, 2000);
    return w.observation_status.ok() && w.result && w.result->state == IoState::COMPLETED &&
           w.result->detail.confirmed_bytes == bytes;
}
}  // namespace

// ---- partial acceptance -------------------------------------------------------

TEST(contract_partial_acceptance_at_every_index) {
    for (long reject = 0; reject < 5; ++reject) {
        Fixture f;
        f.dp.set_reject_at_index(reject);
        IoRequest r[5] = {f.req(0, 512), f.req(512, 512), f.req(1024, 512), f.req(1536, 512), f.req(2048, 512)};
        auto o = f.rt->submit(r, 5, f.ctx());
        CHECK(o.io.has_value());
        CHECK(o.status.code() == StatusCode::BUSY);  // the first rejection's status
        for (long i = 0; i < 5; ++i)
            CHECK(o.initial_states[i].state == (i == reject ? IoRequestState::REJECTED : IoRequestState::ACCEPTED));
        CHECK(completed(*f.rt, *o.io, 4 * 512));
        // the rejected range was not touched
        CHECK(f.buf[reject * 512] == 0 && f.buf[reject * 512 + 511] == 0);
        CHECK(f.rt->release_io(*o.io).ok());
    }
}

TEST(contract_runtime_rejects_before_the_data_path_sees_a_request) {
    Fixture f;
    IoRequest r[4] = {f.req(0, 512), f.req(512, 0), f.req(1 << 16, 512), f.req(1024, 512)};
    r[2].memory_offset = 0;  // target range past the object's end
    auto o = f.rt->submit(r, 4, f.ctx());
    CHECK(o.io.has_value());
    CHECK(o.initial_states[1].status.code() == StatusCode::INVALID_ARGUMENT);  // zero length
    CHECK(o.initial_states[2].status.code() == StatusCode::OUT_OF_RANGE);
    CHECK(o.initial_states[0].state == IoRequestState::ACCEPTED && o.initial_states[3].state == IoRequestState::ACCEPTED);
    CHECK(o.status.code() == StatusCode::INVALID_ARGUMENT);  // the first rejection in input order
    CHECK(completed(*f.rt, *o.io, 1024));
}

TEST(contract_memory_range_checked_against_the_registration) {
    Fixture f;
    IoRequest r[2] = {f.req(0, 512), f.req(0, 512)};
    r[1].memory_offset = (1 << 16) - 256;  // runs past the registered buffer
    auto o = f.rt->submit(r, 2, f.ctx());
    CHECK(o.initial_states[1].status.code() == StatusCode::OUT_OF_RANGE);
    CHECK(completed(*f.rt, *o.io, 512));
}

TEST(contract_every_request_rejected_returns_no_handle) {
    Fixture f;
    f.dp.set_reject_at_index(0);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(!o.io.has_value() && o.status.code() == StatusCode::BUSY);
    CHECK(f.rt->unreleased_terminal_results() == 0);
    // the memory and target hold no in-flight reference afterwards
    CHECK(f.rt->query_memory(f.mem).value().inflight_count == 0);
    CHECK(f.rt->close(f.tgt).ok());
}

TEST(contract_null_request_array_is_invalid) {
    Fixture f;
    auto o = f.rt->submit(nullptr, 2, f.ctx());
    CHECK(!o.io && o.status.code() == StatusCode::INVALID_ARGUMENT && o.initial_states.size() == 2);
}

TEST(contract_mixed_directions_and_targets_in_one_submit) {
    Fixture f;
    auto tb = f.rt->open("mem://b");
    CHECK(tb.ok());
    std::memset(f.buf.data() + 8192, 'w', 512);
    IoRequest r[3] = {f.req(0, 512), IoRequest{IoDirection::WRITE, f.mem, 8192, tb.value(), 1024, 512},
                      IoRequest{IoDirection::READ, f.mem, 4096, tb.value(), 0, 256}};
    auto o = f.rt->submit(r, 3, f.ctx());
    CHECK(o.status.ok() && completed(*f.rt, *o.io, 512 + 512 + 256));
    CHECK((*f.resolver.objects["b"])[1024] == 'w' && (*f.resolver.objects["b"])[1535] == 'w');
    CHECK(f.buf[4096] == 'b' && f.buf[0] == 0);
}

TEST(contract_failed_request_index_is_the_callers_index) {
    Fixture f;
    f.dp.set_reject_at_index(0);  // the DataPath refuses its request 0 ...
    f.dp.set_fail_request(2);     // ... and fails its request 2 (failure indices name DataPath requests)
    IoRequest r[4] = {f.req(0, 512), f.req(512, 512), f.req(1024, 512), f.req(1536, 512)};
    auto o = f.rt->submit(r, 4, f.ctx());
    auto res = f.rt->wait_detail(*o.io, 1000);
    CHECK(res.ok() && res.value().state == IoState::FAILED);
    CHECK(res.value().detail.failure_scope == IoFailureScope::REQUEST_INDICES);
    CHECK(res.value().detail.failed_request_indices.size() == 1);
    CHECK(res.value().detail.failed_request_indices[0] == 2);  // reported in the caller's numbering
    CHECK(res.value().detail.confirmed_bytes == 1024);
}

// ---- IO handle lifecycle -----------------------------------------------------------

TEST(contract_query_tracks_state_and_survives_until_release) {
    Fixture f;
    f.dp.set_manual_mode(true);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(f.rt->query(*o.io).value().state == IoState::IN_FLIGHT);
    f.dp.complete_all();
    CHECK(f.rt->query(*o.io).value().state == IoState::COMPLETED);
    CHECK(f.rt->query(*o.io).value().state == IoState::COMPLETED);  // queries never consume the result
    CHECK(f.rt->release_io(*o.io).ok());
    CHECK(f.rt->query(*o.io).status().code() == StatusCode::NOT_FOUND);
}

TEST(contract_release_of_a_non_terminal_op_is_busy_and_changes_nothing) {
    Fixture f;
    f.dp.set_manual_mode(true);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    for (int i = 0; i < 3; ++i) CHECK(f.rt->release_io(*o.io).code() == StatusCode::BUSY);
    CHECK(f.dp.released == 0);
    f.dp.complete_all();
    CHECK(completed(*f.rt, *o.io, 512));
    CHECK(f.rt->release_io(*o.io).ok() && f.dp.released == 1);
}

TEST(contract_double_release_and_stale_handles_are_not_found) {
    Fixture f;
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(completed(*f.rt, *o.io, 512));
    CHECK(f.rt->release_io(*o.io).ok());
    CHECK(f.rt->release_io(*o.io).code() == StatusCode::NOT_FOUND);
    CHECK(f.rt->wait(*o.io, 10).observation_status.code() == StatusCode::NOT_FOUND);
    // the slot is reused by the next IO with a new generation: the old handle stays dead
    auto o2 = f.rt->submit(r, 1, f.ctx());
    CHECK(o2.io && *o2.io != *o.io);
    CHECK(f.rt->query(*o.io).status().code() == StatusCode::NOT_FOUND);
    CHECK(completed(*f.rt, *o2.io, 512));
}

TEST(contract_wait_zero_timeout_polls) {
    Fixture f;
    f.dp.set_manual_mode(true);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(f.rt->wait(*o.io, 0).observation_status.code() == StatusCode::TIMEOUT);
    f.dp.complete_all();
    CHECK(f.rt->wait(*o.io, 0).observation_status.ok());
}

TEST(contract_wait_result_keeps_the_detail_until_release) {
    Fixture f;
    f.dp.set_fail_request(0);
    IoRequest r[2] = {f.req(0, 512), f.req(512, 512)};
    auto o = f.rt->submit(r, 2, f.ctx());
    auto a = f.rt->wait_result(*o.io, 1000);
    auto b = f.rt->wait_result(*o.io, 1000);
    CHECK(a.result && b.result && a.result->state == IoState::FAILED && b.result->state == IoState::FAILED);
    CHECK(a.result->detail.failed_request_indices == b.result->detail.failed_request_indices);
}

TEST(contract_terminal_budget_counts_failed_results_too) {
    Fixture f(2);
    f.dp.set_fail_request(0);
    IoRequest r[1] = {f.req(0, 512)};
    auto a = f.rt->submit(r, 1, f.ctx());
    CHECK(f.rt->wait(*a.io, 1000).result->state == IoState::FAILED);
    auto b = f.rt->submit(r, 1, f.ctx());
    CHECK(f.rt->wait(*b.io, 1000).observation_status.ok());
    CHECK(f.rt->unreleased_terminal_results() == 2);
    auto c = f.rt->submit(r, 1, f.ctx());
    CHECK(!c.io && c.status.code() == StatusCode::RESOURCE_EXHAUSTED);
    CHECK(c.initial_states[0].status.code() == StatusCode::RESOURCE_EXHAUSTED);
    CHECK(f.rt->release_io(*a.io).ok());
    CHECK(f.rt->unreleased_terminal_results() == 1);
    auto d = f.rt->submit(r, 1, f.ctx());
    CHECK(d.io.has_value());
}

TEST(contract_in_flight_ios_do_not_count_against_the_terminal_budget) {
    Fixture f(1);
    f.dp.set_manual_mode(true);
    IoRequest r[1] = {f.req(0, 512)};
    std::vector<IoHandle> hs;
    for (int i = 0; i < 4; ++i) {
        auto o = f.rt->submit(r, 1, f.ctx());
        CHECK(o.io.has_value());
        hs.push_back(*o.io);
    }
    f.dp.complete_all();
    for (auto& h : hs) CHECK(f.rt->wait(h, 1000).observation_status.ok());
    CHECK(f.rt->unreleased_terminal_results() == 4);
    for (auto& h : hs) CHECK(f.rt->release_io(h).ok());
    CHECK(f.rt->unreleased_terminal_results() == 0);
}

// ---- memory registry ------------------------------------------------------------------

TEST(contract_register_memory_rejects_empty_views) {
    Fixture f;
    MemoryView v;
    v.address = nullptr;
    v.size = 4096;
    CHECK(f.rt->register_memory(v).status().code() == StatusCode::INVALID_ARGUMENT);
    v.address = f.buf.data();
    v.size = 0;
    CHECK(f.rt->register_memory(v).status().code() == StatusCode::INVALID_ARGUMENT);
}

TEST(contract_adjacent_registrations_coexist_overlapping_ones_do_not) {
    Fixture f;
    std::vector<char> other(8192);
    MemoryView a{other.data(), 4096, MemoryKind::HOST}, b{other.data() + 4096, 4096, MemoryKind::HOST};
    auto ha = f.rt->register_memory(a), hb = f.rt->register_memory(b);
    CHECK(ha.ok() && hb.ok() && ha.value() != hb.value());
    MemoryView c{other.data() + 2048, 4096, MemoryKind::HOST};
    CHECK(f.rt->register_memory(c).status().code() == StatusCode::INVALID_ARGUMENT);
    CHECK(f.rt->unregister_memory(ha.value()).ok());
    CHECK(f.rt->register_memory(c).status().code() == StatusCode::INVALID_ARGUMENT);  // still overlaps b
    MemoryView d{other.data(), 2048, MemoryKind::HOST};
    CHECK(f.rt->register_memory(d).ok());  // a's range is free again
}

TEST(contract_query_memory_reports_inflight_references) {
    Fixture f;
    f.dp.set_manual_mode(true);
    IoRequest r[3] = {f.req(0, 512), f.req(512, 512), f.req(1024, 512)};
    auto o = f.rt->submit(r, 3, f.ctx());
    auto info = f.rt->query_memory(f.mem);
    CHECK(info.ok() && info.value().inflight_count == 3 && info.value().size == (1u << 16));
    CHECK(info.value().ownership == MemoryOwnership::CALLER_OWNED && info.value().kind == MemoryKind::HOST);
    f.dp.complete_all();
    CHECK(f.rt->wait(*o.io, 1000).observation_status.ok());
    CHECK(f.rt->query_memory(f.mem).value().inflight_count == 0);
}

TEST(contract_unregister_twice_and_query_after_unregister) {
    Fixture f;
    CHECK(f.rt->unregister_memory(f.mem).ok());
    CHECK(f.rt->unregister_memory(f.mem).code() == StatusCode::NOT_FOUND);
    CHECK(f.rt->query_memory(f.mem).status().code() == StatusCode::NOT_FOUND);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(!o.io && o.initial_states[0].status.code() == StatusCode::NOT_FOUND);
}

TEST(contract_allocate_and_free_runtime_owned_host_memory) {
    Fixture f;
    MemorySpec spec;
    spec.size = 1 << 20;
    spec.kind = MemoryKind::HOST;
    auto a = f.rt->allocate_memory(spec);
    CHECK(a.ok() && a.value().address && a.value().size == (1u << 20));
    CHECK(f.rt->query_memory(a.value().handle).value().ownership == MemoryOwnership::RUNTIME_OWNED);
    // usable as IO memory like any registration
    IoRequest r[1] = {IoRequest{IoDirection::READ, a.value().handle, 0, f.tgt, 0, 4096}};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(completed(*f.rt, *o.io, 4096));
    CHECK(static_cast<char*>(a.value().address)[7] == static_cast<char>(49));
    CHECK(f.rt->release_io(*o.io).ok());
    CHECK(f.rt->unregister_memory(a.value().handle).ok() || true);
    spec.size = 0;
    CHECK(f.rt->allocate_memory(spec).status().code() == StatusCode::INVALID_ARGUMENT);
}

TEST(contract_free_memory_refuses_caller_owned_memory) {
    Fixture f;
    CHECK(f.rt->free_memory(f.mem).code() == StatusCode::INVALID_ARGUMENT);
    CHECK(f.rt->query_memory(f.mem).ok());  // still registered
}

// ---- targets ------------------------------------------------------------------------------

TEST(contract_query_target_reports_size_path_and_inflight) {
    Fixture f;
    auto info = f.rt->query_target(f.tgt);
    CHECK(info.ok() && info.value().logical_size == (1u << 16) && info.value().data_path_key == "mock");
    CHECK(info.value().uri == "mem://a");
    f.dp.set_manual_mode(true);
    IoRequest r[2] = {f.req(0, 512), f.req(512, 512)};
    auto o = f.rt->submit(r, 2, f.ctx());
    CHECK(f.rt->query_target(f.tgt).value().inflight_count == 2);
    f.dp.complete_all();
    CHECK(f.rt->wait(*o.io, 1000).observation_status.ok());
    CHECK(f.rt->query_target(f.tgt).value().inflight_count == 0);
}

TEST(contract_open_unknown_scheme_or_object_fails_cleanly) {
    Fixture f;
    CHECK(!f.rt->open("nfs://x").ok());
    CHECK(f.rt->open("mem://missing").status().code() == StatusCode::NOT_FOUND);
    CHECK(!f.rt->open("no-scheme").ok());
    CHECK(f.rt->open("mem://a").ok());  // the runtime keeps serving afterwards
}

TEST(contract_close_batch_closes_valid_handles_and_reports_the_first_error) {
    Fixture f;
    auto b = f.rt->open("mem://b");
    CHECK(b.ok());
    TargetHandle stale = f.tgt;
    CHECK(f.rt->close(stale).ok());
    auto st = f.rt->close_batch({b.value(), stale});
    CHECK(st.code() == StatusCode::NOT_FOUND);
    CHECK(f.rt->query_target(b.value()).status().code() == StatusCode::NOT_FOUND);  // b was closed
}

TEST(contract_reopened_target_gets_a_new_handle_and_the_old_one_dies) {
    Fixture f;
    const TargetHandle old = f.tgt;
    CHECK(f.rt->close(old).ok());
    auto n = f.rt->open("mem://a");
    CHECK(n.ok() && n.value() != old);
    IoRequest r[1] = {IoRequest{IoDirection::READ, f.mem, 0, old, 0, 512}};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(!o.io && o.initial_states[0].status.code() == StatusCode::NOT_FOUND);
    r[0].target = n.value();
    o = f.rt->submit(r, 1, f.ctx());
    CHECK(o.io && completed(*f.rt, *o.io, 512));
}

TEST(contract_open_batch_of_many_uris_keeps_input_order) {
    Fixture f;
    std::vector<std::string> uris;
    for (int i = 0; i < 100; ++i) uris.push_back(i % 10 == 9 ? "mem://missing" : (i % 2 ? "mem://a" : "mem://b"));
    auto v = f.rt->open_batch(uris);
    CHECK(v.size() == 100);
    for (int i = 0; i < 100; ++i) {
        if (i % 10 == 9) {
            CHECK(!v[i].ok());
            continue;
        }
        CHECK(v[i].ok());
        CHECK(f.rt->query_target(v[i].value()).value().uri == uris[i]);
    }
}

TEST(contract_data_path_target_maps_handles) {
    Fixture f;
    auto d = f.rt->data_path_target(f.tgt);
    CHECK(d.ok());
    CHECK(f.rt->close(f.tgt).ok());
    CHECK(f.rt->data_path_target(f.tgt).status().code() == StatusCode::NOT_FOUND);
}

// ---- lifecycle ----------------------------------------------------------------------------

TEST(contract_everything_refuses_after_shutdown) {
    Fixture f;
    CHECK(f.rt->shutdown(1000).ok());
    CHECK(f.rt->shutdown(1000).ok());  // idempotent
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(!o.io && o.status.code() == StatusCode::NOT_READY);
    auto v = f.rt->open_batch({"mem://a", "mem://b"});
    CHECK(v.size() == 2 && v[0].status().code() == StatusCode::NOT_READY && v[1].status().code() == StatusCode::NOT_READY);
    CHECK(f.rt->open("mem://a").status().code() == StatusCode::NOT_READY);
}

TEST(contract_shutdown_waits_for_inflight_then_releases_them) {
    Fixture f;
    f.dp.set_manual_mode(true);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    std::thread finisher([&] {
        std::this_thread::sleep_for(std::chrono::milliseconds(30));
        f.dp.complete_all();
    });
    CHECK(f.rt->shutdown(2000).ok());
    finisher.join();
    CHECK(f.dp.released >= 1 && f.dp.shut_down);
    CHECK(f.rt->state() == RuntimeState::STOPPED);
}

TEST(contract_shutdown_past_its_deadline_keeps_pending_ops_and_can_be_retried) {
    Fixture f;
    f.dp.set_manual_mode(true);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(o.io.has_value());
    auto st = f.rt->shutdown(20);
    CHECK(st.code() == StatusCode::TIMEOUT);
    CHECK(f.rt->state() == RuntimeState::DRAINING && !f.dp.shut_down);
    // draining: no new work, the pending op stays observable and completes normally
    auto o2 = f.rt->submit(r, 1, f.ctx());
    CHECK(!o2.io && o2.status.code() == StatusCode::NOT_READY);
    CHECK(f.rt->query(*o.io).value().state == IoState::IN_FLIGHT);
    f.dp.complete_all();
    CHECK(completed(*f.rt, *o.io, 512));
    CHECK(f.rt->shutdown(1000).ok());
    CHECK(f.rt->state() == RuntimeState::STOPPED && f.dp.shut_down);
}

TEST(contract_close_and_unregister_wait_for_the_io_that_uses_them) {
    Fixture f;
    f.dp.set_manual_mode(true);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(f.rt->close(f.tgt).code() == StatusCode::BUSY);
    CHECK(f.rt->unregister_memory(f.mem).code() == StatusCode::BUSY);
    CHECK(f.rt->query_target(f.tgt).ok());  // the refused close changed nothing
    f.dp.complete_all();
    CHECK(completed(*f.rt, *o.io, 512));
    // a terminal op no longer holds them, released or not
    CHECK(f.rt->close(f.tgt).ok());
    CHECK(f.rt->unregister_memory(f.mem).ok());
    CHECK(f.rt->release_io(*o.io).ok());
}

TEST(contract_failed_progress_does_not_lose_the_op) {
    Fixture f;
    f.dp.set_manual_mode(true);
    f.dp.set_fail_progress(true);
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(f.rt->wait(*o.io, 5).observation_status.code() == StatusCode::TIMEOUT);
    f.dp.set_fail_progress(false);
    f.dp.complete_all();
    CHECK(completed(*f.rt, *o.io, 512));
}

TEST(contract_enqueue_wait_needs_a_device_completion_data_path) {
    Fixture f;
    IoRequest r[1] = {f.req(0, 512)};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(f.rt->enqueue_wait(&*o.io, 1, nullptr).code() == StatusCode::UNSUPPORTED);
    IoHandle bogus;
    CHECK(f.rt->enqueue_wait(&bogus, 1, nullptr).code() == StatusCode::NOT_FOUND);
}

TEST(contract_capabilities_and_device_queries) {
    Fixture f;
    auto caps = f.rt->data_path_capabilities();
    CHECK(caps.size() == 1 && caps[0].name == "mock");
    CHECK(f.rt->accel_id() == 0);
    CHECK(f.rt->state() == RuntimeState::RUNNING);
}

TEST(contract_create_refuses_duplicate_bindings) {
    MemResolver res;
    MockDataPath a, b;
    RuntimeConfig c;
    RuntimeComponents comps;
    comps.resolvers.push_back({"mem", &res});
    comps.resolvers.push_back({"mem", &res});
    comps.data_paths.push_back({"mock", &a, DataPathConfig{"mock"}});
    CHECK(StorageRuntime::create(c, comps).status().code() == StatusCode::INVALID_ARGUMENT);
    comps.resolvers.pop_back();
    comps.data_paths.push_back({"mock", &b, DataPathConfig{"mock"}});
    CHECK(StorageRuntime::create(c, comps).status().code() == StatusCode::INVALID_ARGUMENT);
    comps.data_paths.pop_back();
    comps.data_paths.push_back({"", &b, DataPathConfig{""}});
    CHECK(StorageRuntime::create(c, comps).status().code() == StatusCode::INVALID_ARGUMENT);
}

TEST(contract_runtimes_do_not_accept_each_others_handles) {
    Fixture f, g;
    IoRequest r[1] = {IoRequest{IoDirection::READ, f.mem, 0, g.tgt, 0, 512}};
    auto o = f.rt->submit(r, 1, f.ctx());
    CHECK(!o.io && o.initial_states[0].status.code() == StatusCode::NOT_FOUND);
    CHECK(g.rt->close(f.tgt).code() == StatusCode::NOT_FOUND);
    CHECK(g.rt->unregister_memory(f.mem).code() == StatusCode::NOT_FOUND);
}

// ---- concurrency ----------------------------------------------------------------------------

TEST(contract_concurrent_submitters_and_waiters) {
    Fixture f(1024);
    std::atomic<int> bad{0};
    std::vector<std::thread> th;
    for (int t = 0; t < 8; ++t)
        th.emplace_back([&, t] {
            for (int i = 0; i < 50; ++i) {
                const std::uint64_t off = (static_cast<std::uint64_t>(t) * 50 + i) % 64 * 1024;
                IoRequest r[2] = {f.req(off, 512), f.req(off + 512, 512)};
                auto o = f.rt->submit(r, 2, host_ctx());
                if (!o.io || !completed(*f.rt, *o.io, 1024) || !f.rt->release_io(*o.io).ok()) ++bad;
            }
        });
    for (auto& x : th) x.join();
    CHECK(bad.load() == 0);
    CHECK(f.rt->unreleased_terminal_results() == 0);
    CHECK(f.rt->query_memory(f.mem).value().inflight_count == 0);
}

TEST(contract_concurrent_open_close_and_submit) {
    Fixture f(1024);
    std::atomic<int> bad{0};
    std::thread opener([&] {
        for (int i = 0; i < 200; ++i) {
            auto h = f.rt->open("mem://b");
            if (!h.ok() || !f.rt->close(h.value()).ok()) ++bad;
        }
    });
    for (int i = 0; i < 200; ++i) {
        IoRequest r[1] = {f.req((i % 64) * 512, 512)};
        auto o = f.rt->submit(r, 1, f.ctx());
        if (!o.io || !completed(*f.rt, *o.io, 512) || !f.rt->release_io(*o.io).ok()) ++bad;
    }
    opener.join();
    CHECK(bad.load() == 0);
}
