"""Population sharding host logic on world-size-2 gloo ranks (CPU).

Each rank evaluates its own antithetic pairs with the CPU oracle on a tiny
hybrid configuration; the all-gathered fitness must equal a single-process
evaluation of the whole population.  A rank that drops out must make the
survivor's collective fail within the process-group timeout (no hang)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ennx_b200.model import HybridConfig
from ennx_b200.population import PopulationStep, shard_pairs

TINY = HybridConfig(layers=2, hidden=256, vocab=300, attn_period=2, q_heads=2, kv_heads=1, kda_heads=1,
                    gate_rank=64, experts=4, top_k=2, expert_width=128)


def test_shard_pairs_cover_population():
    for pairs in (1, 5, 16):
        for world in (1, 2, 4, 8):
            got = [shard_pairs(pairs, world, r) for r in range(world)]
            covered = [p for f, c in got for p in range(f, f + c)]
            assert covered == list(range(pairs))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    import oracle as O
    rng = np.random.default_rng(0)
    w = {"embedding": O.to_bf16_bits(rng.standard_normal((TINY.vocab, TINY.hidden)).astype(np.float32) * 0.05),
         "final_norm": O.to_bf16_bits(np.ones(TINY.hidden, np.float32)), "layers": []}
    for l in range(TINY.layers):
        L = {}
        for name, shp in TINY.layer_shapes(l).items():
            if name in ("attn_norm", "moe_norm", "out_norm"):
                L[name] = O.to_bf16_bits(np.ones(shp, np.float32))
            elif name in ("decay", "time_bias"):
                L[name] = O.to_bf16_bits(np.zeros(shp, np.float32))
            else:
                L[name] = O.to_bf16_bits(rng.standard_normal(shp).astype(np.float32) * 0.05)
        w["layers"].append(L)
    return w


def _cpu_evaluator(w):
    from oracle import forward as OF

    def evaluate(tokens, seed, sigma, first, count):
        return torch.tensor(OF.population_forward(TINY, w, tokens.numpy(), seed, sigma, first, count),
                            dtype=torch.float32)
    return evaluate


def _cpu_update(w, log):
    from oracle import forward as OF

    def coefficients(fitness, sigma, lr, pairs):
        import oracle as O
        return torch.from_numpy(O.es_coefficients(fitness.numpy(), sigma, lr, pairs))

    def update(seed, coef):
        new = OF.population_update(TINY, w, seed, coef.numpy())
        w.update(new)
        log.append((seed, coef.numpy().copy()))
    return coefficients, update


def _worker(rank, world, port, out_q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        w = _weights()
        tok = torch.from_numpy(np.random.default_rng(1).integers(0, TINY.vocab, (1, 17)).astype(np.int32))
        log = []
        coefficients, update = _cpu_update(w, log)
        step = PopulationStep(_cpu_evaluator(w), num_pairs=2, sigma=0.02, lr=0.1,
                              coefficients=coefficients if rank == 0 else (lambda *a: None), update=update)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the exchange")
        res = step(tok, seed=5)
        out_q.put((rank, "ok", res.fitness.numpy().tolist(), res.next_seed, res.coefficients.numpy().tolist(),
                   w["layers"][0]["w_qkv"].tobytes()))
    except RuntimeError as e:
        out_q.put((rank, "error", str(e), None, None, None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results)


def test_two_gloo_ranks_match_single_process():
    res = _run(2)
    assert [r[1] for r in res] == ["ok", "ok"]
    assert res[0][2] == res[1][2] and res[0][3] == res[1][3] == 6
    w = _weights()
    single = _cpu_evaluator(w)(
        torch.from_numpy(np.random.default_rng(1).integers(0, TINY.vocab, (1, 17)).astype(np.int32)), 5, 0.02, 0, 2)
    np.testing.assert_allclose(res[0][2], single.numpy(), rtol=0, atol=0)
    # rank 0's coefficients reached rank 1 unchanged, and both replicas moved
    # identically: the update of the gathered fitness, regenerated locally
    import oracle as O
    from oracle import forward as OF
    coef = O.es_coefficients(single.numpy(), 0.02, 0.1)
    assert res[0][4] == res[1][4] == coef.tolist()
    expect = OF.population_update(TINY, w, 5, coef)["layers"][0]["w_qkv"].tobytes()
    assert res[0][5] == res[1][5] == expect


def test_rank_failure_surfaces_as_error_not_hang():
    res = _run(2, fail_rank=1)
    status = {r[0]: r[1] for r in res}
    assert status[1] == "error"
    assert status[0] == "error"  # the survivor's all_gather times out / is aborted


def test_resident_es_state_round_rules():
    """ask/tell bookkeeping of ResidentEsState (single process, CPU oracle)."""
    from ennx_b200.population import ResidentEsState
    w = _weights()
    log = []
    coefficients, update = _cpu_update(w, log)
    step = PopulationStep(_cpu_evaluator(w), num_pairs=2, sigma=0.02, lr=0.1, coefficients=coefficients,
                          update=update)
    state = ResidentEsState(step, seed=11)
    tok = torch.from_numpy(np.random.default_rng(2).integers(0, TINY.vocab, (1, 9)).astype(np.int32))
    r, f = state.ask_evaluate(tok)
    assert r.seed == 11 and state.seed == 12 and len(log) == 1 and log[0][0] == 11
    r2 = state.ask()
    with pytest.raises(ValueError, match="tell must finish the resident forward round before ask"):
        state.ask()
    with pytest.raises(ValueError, match="does not match pending trial"):
        state.tell(type(r2)(99, r2.step), f)
    state.tell(r2, f)
    with pytest.raises(ValueError, match="no resident forward round is pending"):
        state.tell(r2, f)
    with pytest.raises(ValueError, match="learning rate"):
        ResidentEsState(PopulationStep(_cpu_evaluator(w), num_pairs=2, sigma=0.02))
