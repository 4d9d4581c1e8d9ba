"""Host emulation of the NVLink collectives' flag protocols (race detection
without a GPU): randomized CTA interleavings across and within ranks must
never read a stale or overwritten slot, write a slot someone may still
read, or deadlock; deliberately broken variants must be caught."""
import pytest

from rlx_models_b200.parallel import protocol_sim as ps


@pytest.mark.parametrize("mode", ["pull", "two_shot", "mixed"])
@pytest.mark.parametrize("world,M", [(2, 1), (2, 5), (4, 3), (4, 8), (8, 2), (8, 8)])
def test_tp_decode_allreduce_protocols(mode, world, M):
    for seed in range(12):
        ps.tp_decode_ops(world, M, n_ops=5, seed=seed, rows=8, mode=mode)


@pytest.mark.parametrize("world,R", [(2, 1), (2, 4), (4, 3), (8, 2)])
def test_tp_argmax_protocol(world, R):
    for seed in range(20):
        ps.tp_argmax_ops(world, R, n_ops=5, seed=seed)


def test_emulator_catches_single_buffered_argmax_keys():
    """With one key buffer a fast rank's next op pushes its key into a slot
    whose previous key a slow peer has not read yet."""
    caught = 0
    for seed in range(40):
        try:
            ps.tp_argmax_ops(4, 2, n_ops=6, seed=seed, buffers=1)
        except ps.ProtocolError:
            caught += 1
    assert caught > 0


def test_emulator_catches_single_buffered_accumulator(monkeypatch):
    """Accumulating every op into the same parity (no double buffering) lets a
    fast rank's next GEMM overwrite a partial a slow peer is still reading."""
    orig = ps.gemm_acc

    def gemm_same_parity(sim, rank, op, par, M):
        return orig(sim, rank, op, 0, M)

    def pull_same_parity(sim, rank, op, par, M, rows):
        W = sim.world

        def cta(i):
            def g():
                m = sim.mem(rank)
                e = m["ctr1"]["epoch"] + 1
                if i == 0:
                    for q in range(W):
                        sim.mem(q)["flags"][rank] = e
                        yield
                yield ps.Wait(lambda: all(f >= e for f in m["flags"]))
                for q in range(W):
                    v = sim.mem(q)["acc"][0][i]
                    ps._check(v == op, f"rank {rank} op {op}: stale {v}")
                    yield
                m["acc"][0][i] = ps.ZERO  # clears the slot it just used: peers may still be reading it
                yield
                m["ctr1"]["dep"] += 1
                if m["ctr1"]["dep"] == M:
                    m["ctr1"]["dep"] = 0
                    m["ctr1"]["epoch"] = e
            return g
        sim.launch(rank, f"pull{op}", [cta(i) for i in range(M)])

    monkeypatch.setattr(ps, "gemm_acc", gemm_same_parity)
    monkeypatch.setattr(ps, "ar_pull", pull_same_parity)
    caught = 0
    for seed in range(40):
        try:
            ps.tp_decode_ops(4, 4, n_ops=4, seed=seed, rows=4, mode="pull")
        except ps.ProtocolError:
            caught += 1
    assert caught > 0


def test_emulator_catches_missing_second_barrier(monkeypatch):
    """A two-shot kernel whose copy phase does not wait for the owners' result
    flags reads rows that are not written yet."""
    def ar2_no_barrier2(sim, rank, op, par, M, rows):
        W = sim.world
        rpr = -(-M // W)
        n_my = max(0, min(rpr, M - rank * rpr))

        def cta(i):
            def g():
                m = sim.mem(rank)
                e = m["ctr2"]["epoch"] + 1
                if i == 0:
                    for q in range(W):
                        sim.mem(q)["flags2"][0][rank] = e
                        yield
                if i < n_my:
                    yield ps.Wait(lambda: all(f >= e for f in m["flags2"][0]))
                    yield
                    m["res"][i] = op
                if i < M:
                    owner, j = i // rpr, i % rpr
                    v = sim.mem(owner)["res"].get(j)
                    ps._check(v == op, f"rank {rank} op {op}: copied {v}")
                yield
                m["ctr2"]["dep"] += 1
                if m["ctr2"]["dep"] == max(M, rows):
                    m["ctr2"]["dep"] = 0
                    m["ctr2"]["epoch"] = e
            return g
        sim.launch(rank, f"ar2_{op}", [cta(i) for i in range(max(M, rows))])

    monkeypatch.setattr(ps, "ar2", ar2_no_barrier2)
    with pytest.raises(ps.ProtocolError):
        for seed in range(40):
            ps.tp_decode_ops(4, 8, n_ops=3, seed=seed, rows=8, mode="two_shot")


def test_emulator_reports_deadlock():
    sim = ps.Sim(2, 0)

    def waits_forever():
        yield ps.Wait(lambda: False)

    sim.launch(0, "k", [waits_forever])
    with pytest.raises(ps.ProtocolError, match="deadlock"):
        sim.run()
