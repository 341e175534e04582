"""Multi-GPU tests (one process per GPU, NCCL process group for the bootstrap), at
world sizes 2, 4 and 8 (each skipped when the box has fewer GPUs):

* the peer-memory reductions are bit-exact against the oracle in every wire mode and
  both protocols, including the [32768, 2048] int8 out_proj site of the 1.4b bench
  (two-shot at 4 and 8 ranks) with 1% outlier channels, and every rank holds the
  same bytes (the reference's cross-rank bit identity, tests/test_per_site_allreduce.py);
* the TP model matches the oracle's TP emulation at the same world size with identical
  results on every rank, graphed decode equals eager decode bitwise, and the persistent
  decode kernel agrees with the per-layer chain;
* the vocabulary-parallel lm_head gives the replicated lm_head's logits and greedy tokens,
  bitwise; so does the x_proj GEMM with AllReduce #1 in its epilogue against the GEMM
  followed by the reduction kernel;
* the out_proj epilogue gives the same bits through one-shot, two-shot and capped grids,
  and the overlapped micro-batch prefill equals the serial prefill bitwise.

One spawn per world size runs every check (``_suite``); large results travel back as
SHA-256 digests.  Two more tests, at 2 GPUs, make a reduction and a decode step wait
for a peer that never arrives and check the timeout status (bounded waits)."""
import datetime
import hashlib
import os
import tempfile

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
WS_LIST = (2, 4, 8)
BIG = (32768, 2048)  # the 1.4b out_proj site of a 32 x 1024 prefill


def _ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def needs(ws):
    return pytest.mark.skipif(_ngpu() < ws, reason=f"needs {ws} GPUs")


def _init(rank, init_file, ws):
    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))


def _finish():
    import torch.distributed as dist

    from mamba_tp_lite_b200.tp_utils import destroy_comms

    torch.cuda.synchronize()
    dist.barrier()
    destroy_comms()
    dist.barrier()
    dist.destroy_process_group()


def _spawn(fn, ws, *args, timeout=600):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=fn, args=(r, os.path.join(d, "rdv"), q, ws) + args) for r in range(ws)]
        for p in procs:
            p.start()
        try:
            res = dict(q.get(timeout=timeout) for _ in range(ws))
        finally:
            for p in procs:
                p.join(timeout=60)
                if p.is_alive():
                    p.kill()
    for r in range(ws):
        if isinstance(res[r], str):
            raise AssertionError(f"rank {r}: {res[r]}")
    return res


def _digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


def _partial(rank, rows, cols, outliers=False):
    """The seeded partial of one rank: N(0, 3^2); with outliers, a fixed 1% of the
    columns scaled by 20 (the activation model of the collective microbench)."""
    x = torch.randn(rows, cols, generator=torch.Generator().manual_seed(1000 * rank + rows)) * 3
    if outliers:
        idx = torch.randperm(cols, generator=torch.Generator().manual_seed(77))[:max(1, cols // 100)]
        x[:, idx] *= 20
    return x


RED_CASES = ((1, 160), (33, 2048), (4096, 768), (20000, 2048), (7, 18))


# ------------------------------------------------------------------ one spawn per world size
def _suite(rank, init_file, q, ws):
    try:
        _init(rank, init_file, ws)
        from mamba_tp_lite_b200 import _lib as L
        from mamba_tp_lite_b200.checkpoint import random_init_state_dict
        from mamba_tp_lite_b200.config import MambaConfig
        from mamba_tp_lite_b200.cuda_graph import GraphedStepper
        from mamba_tp_lite_b200.tp_model import TPMambaLM
        from mamba_tp_lite_b200.tp_utils import build_spec, get_comm

        out = {"reduce": {}, "model": {}, "proto": {}, "overlap": {}}
        # ---- raw reductions: every mode, default and forced two-shot protocol
        for protocol in (None, "twoshot"):
            if protocol:
                os.environ["MTP_COMM_PROTOCOL"] = protocol
            cases = RED_CASES + ((BIG[0], BIG[1], True),)
            for case in cases:
                rows, cols = case[:2]
                big = len(case) == 3
                comm = get_comm(None, rank, ws, cols, cols)
                x = _partial(rank, rows, cols, outliers=big).cuda()
                for mode in ((L.RED_INT8TOK,) if big else (L.RED_FP32, L.RED_FP16, L.RED_INT8TOK, L.RED_INT8TENSOR,
                                                             L.RED_INT8SUM, L.RED_INT8LEGACY)):
                    y = torch.empty_like(x)
                    for _ in range(2):  # back-to-back calls on one site
                        L.call("mtp_allreduce", comm.ptr, 1, mode, L.ptr(x), L.ptr(y), rows, cols, L.stream_ptr())
                    torch.cuda.synchronize()
                    out["reduce"][(protocol, rows, cols, mode)] = _digest(y.cpu().numpy())
                comm.check()
                del x, y
            os.environ.pop("MTP_COMM_PROTOCOL", None)
        torch.cuda.empty_cache()
        # ---- TP model: fp32 and bf16, three wire maps, eager / graphed / per-layer chain decode
        cfg = MambaConfig(d_model=256, n_layer=3, vocab_size=1000, dt_rank=16)
        ids = torch.randint(0, cfg.vocab_size, (2, 72), generator=torch.Generator().manual_seed(4))
        for dtype in (torch.float32, torch.bfloat16):
            sd = random_init_state_dict(cfg, seed=3, dtype=dtype)
            for spec in ("fp32", "fp16", "int8"):
                m = TPMambaLM.from_state_dict_shard(cfg, sd, rank, ws, dtype=dtype, allreduce_dtype=spec,
                                                    device="cuda")
                logits, cache = m.prefill(ids.cuda())
                nxt = torch.zeros(2, 1, dtype=torch.long, device="cuda")
                eager = [m.step(nxt, cache).clone() for _ in range(3)]
                _, cg = m.prefill(ids.cuda())
                st = GraphedStepper(m, cg, 2, "cuda")
                st.capture()
                graphed = [st.replay(nxt).clone() for _ in range(3)]
                st.release()
                count = m.layers[0].mixer.comm.count
                os.environ["MTP_DECODE_FUSED"] = "0"  # the same steps through the per-layer chain
                _, cc = m.prefill(ids.cuda())
                chain = [m.step(nxt, cc).float().cpu().numpy() for _ in range(3)]
                os.environ.pop("MTP_DECODE_FUSED")
                out["model"][(str(dtype), spec)] = (
                    logits.float().cpu().numpy(), [e.float().cpu().numpy() for e in eager],
                    all(torch.equal(a, b) for a, b in zip(eager, graphed)), count, chain,
                    getattr(m, "_mtp_decode", None) is not None)
                del m
        # ---- per-tensor-scale variants mixed with per-row sites (sequence-parallel epilogue off)
        sd = random_init_state_dict(cfg, seed=12, dtype=torch.float32)
        vspec = build_spec({"default": "int8", "overrides": {"0:out_proj": "int8_sum", "1:x_proj": "int8_gather",
                                                             "2:out_proj": "int8_legacy", "2:x_proj": "int8_sum",
                                                             "1:out_proj": "fp16"}}, cfg.n_layer)
        m = TPMambaLM.from_state_dict_shard(cfg, sd, rank, ws, dtype=torch.float32, allreduce_dtype=vspec,
                                            device="cuda")
        lg, cache = m.prefill(ids.cuda())
        st = m.step(torch.full((2, 1), 5, dtype=torch.long, device="cuda"), cache)
        out["variants"] = (lg.float().cpu().numpy(), st.float().cpu().numpy(), m.layers[0].mixer.comm.count)
        del m
        # ---- vocabulary-parallel lm_head (default up to 256 rows) == replicated lm_head, bitwise
        out["vocab"] = {}
        for dtype in (torch.float32, torch.bfloat16):
            sd = random_init_state_dict(cfg, seed=5, dtype=dtype)
            m = TPMambaLM.from_state_dict_shard(cfg, sd, rank, ws, dtype=dtype, allreduce_dtype="int8", device="cuda")
            for vp in ("0", "256"):
                os.environ["MTP_VOCAB_PARALLEL_ROWS"] = vp
                lg, cache = m.prefill(ids.cuda())                       # 144 rows
                lg1, _ = m.prefill(ids[:1, :20].cuda())                 # 20 rows
                st = m.step(torch.full((2, 1), 7, dtype=torch.long, device="cuda"), cache)  # 2 rows
                toks = m.generate(ids[:, :9].cuda(), 4, graphed=True)   # graphed greedy decode
                out["vocab"][(str(dtype), vp)] = (_digest(lg.float().cpu().numpy()),
                                                  _digest(lg1.float().cpu().numpy()),
                                                  _digest(st.float().cpu().numpy()), toks.cpu().numpy())
            os.environ.pop("MTP_VOCAB_PARALLEL_ROWS")
            del m
        # ---- x_proj GEMM with AllReduce #1 in its epilogue == GEMM + reduction kernel, bitwise
        out["xfused"] = {}
        sd = random_init_state_dict(cfg, seed=6, dtype=torch.bfloat16)
        spec = build_spec({"default": "int8", "overrides": {"1:x_proj": "fp32", "2:x_proj": "fp16"}}, cfg.n_layer)
        m = TPMambaLM.from_state_dict_shard(cfg, sd, rank, ws, dtype=torch.bfloat16, allreduce_dtype=spec,
                                            device="cuda")
        ids3 = torch.randint(0, cfg.vocab_size, (4, 520), generator=torch.Generator().manual_seed(11)).cuda()
        for fz in ("0", "1"):  # "1" forces the epilogue form at every world size
            os.environ["MTP_XPROJ_FUSED"] = fz
            lg, cache = m.prefill(ids3)
            out["xfused"][fz] = (_digest(lg.float().cpu().numpy()),
                                 [_digest(lc.ssm_state.cpu().numpy()) for lc in cache.layers])
        os.environ.pop("MTP_XPROJ_FUSED")
        get_comm(None, rank, ws, cfg.dt_rank + 2 * cfg.d_state, cfg.d_model).check()
        del m
        # ---- out_proj epilogue through one-shot, two-shot and a capped grid
        rows, d = 3000, 1024
        comm = get_comm(None, rank, ws, 48, d)
        part = torch.randn(rows, d, generator=torch.Generator().manual_seed(7 + rank)).cuda() * 2
        w = torch.randn(d, generator=torch.Generator().manual_seed(9)).cuda().to(torch.bfloat16)
        own = np.arange(rank, rows, ws)  # the sequence-parallel epilogue's rows of this rank (r % ws)
        for proto in ("oneshot", "twoshot", "capped", "sp"):
            os.environ["MTP_COMM_PROTOCOL"] = "oneshot" if proto == "capped" else proto
            os.environ["MTP_COMM_SP"] = "1" if proto == "sp" else "0"
            comm.set_max_ctas(16 if proto == "capped" else 0)
            for mode in (L.RED_FP32, L.RED_FP16, L.RED_INT8TOK):
                resid = torch.ones(rows, d, device="cuda")
                normed = torch.empty(rows, d, device="cuda", dtype=torch.bfloat16)
                L.call("mtp_reduce_outproj", comm.ptr, mode, L.ptr(part), rows, d, None, L.ptr(resid), L.ptr(w),
                       1e-5, L.ptr(normed), L.BF16, L.stream_ptr())
                torch.cuda.synchronize()
                r_np = resid.cpu().numpy()
                out["proto"][(proto, mode)] = (_digest(r_np), _digest(normed.float().cpu().numpy()),
                                               _digest(r_np[own]))
        comm.set_max_ctas(0)
        os.environ.pop("MTP_COMM_PROTOCOL")
        os.environ.pop("MTP_COMM_SP")
        comm.check()
        # ---- overlapped micro-batch prefill == serial prefill
        sd = random_init_state_dict(cfg, seed=8, dtype=torch.bfloat16)
        spec = build_spec({"default": "int8", "overrides": {"0:out_proj": "fp16", "1:x_proj": "fp32"}}, cfg.n_layer)
        m = TPMambaLM.from_state_dict_shard(cfg, sd, rank, ws, dtype=torch.bfloat16, allreduce_dtype=spec,
                                            device="cuda")
        ids2 = torch.randint(0, cfg.vocab_size, (5, 520), generator=torch.Generator().manual_seed(9)).cuda()
        for mode in ("1", "0"):
            os.environ["MTP_PREFILL_OVERLAP"] = mode
            c0 = m.layers[0].mixer.comm.count
            lg, cache = m.prefill(ids2)
            lg2, _ = m.prefill(ids2[:, :7], cache)  # chunked continuation from the overlapped cache
            out["overlap"][mode] = (lg.float().cpu().numpy(), lg2.float().cpu().numpy(),
                                    [(lc.conv_state.float().cpu().numpy(), lc.ssm_state.cpu().numpy())
                                     for lc in cache.layers], m.layers[0].mixer.comm.count - c0)
        os.environ.pop("MTP_PREFILL_OVERLAP")
        q.put((rank, out))
        _finish()
    except Exception as e:  # report instead of hanging the parent
        import traceback

        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


_RESULTS = {}


def suite(ws):
    if ws not in _RESULTS:
        _RESULTS[ws] = _spawn(_suite, ws)
    return _RESULTS[ws]


# ------------------------------------------------------------------ raw reductions
@pytest.mark.parametrize("ws", WS_LIST)
def test_peer_reductions_bit_exact_vs_oracle(ws):
    if _ngpu() < ws:
        pytest.skip(f"needs {ws} GPUs")
    from mamba_tp_lite_b200 import _lib as L
    from oracle import mamba_oracle as O

    res = suite(ws)
    names = {L.RED_FP32: "fp32", L.RED_FP16: "fp16", L.RED_INT8TOK: "int8", L.RED_INT8TENSOR: "int8_gather",
             L.RED_INT8SUM: "int8_sum", L.RED_INT8LEGACY: "int8_legacy"}
    want_cache = {}
    for (protocol, rows, cols, mode), got in res[0]["reduce"].items():
        key = (rows, cols, mode)
        if key not in want_cache:
            big = (rows, cols) == BIG
            xs = [_partial(r, rows, cols, outliers=big).numpy() for r in range(ws)]
            want_cache[key] = _digest(O.REDUCE_FNS[names[mode]](xs))
            del xs
        assert got == want_cache[key], (protocol, rows, cols, names[mode])
        for r in range(1, ws):  # every rank holds the same bytes
            assert res[r]["reduce"][(protocol, rows, cols, mode)] == got, (r, protocol, rows, cols)


# ------------------------------------------------------------------ TP model
@pytest.mark.parametrize("ws", WS_LIST)
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_tp_model_matches_oracle_and_ranks_agree(ws, dtype_name):
    if _ngpu() < ws:
        pytest.skip(f"needs {ws} GPUs")
    from mamba_tp_lite_b200.checkpoint import random_init_state_dict
    from mamba_tp_lite_b200.config import MambaConfig
    from oracle import mamba_oracle as O

    res = suite(ws)
    dtype = getattr(torch, dtype_name)
    cfg = MambaConfig(d_model=256, n_layer=3, vocab_size=1000, dt_rank=16)
    sd = random_init_state_dict(cfg, seed=3, dtype=dtype)
    ids = torch.randint(0, cfg.vocab_size, (2, 72), generator=torch.Generator().manual_seed(4)).numpy()
    for spec in ("fp32", "fp16", "int8"):
        lg0, st0, graph_ok, count, chain0, fused = res[0]["model"][(str(dtype), spec)]
        assert fused == (dtype_name == "bfloat16"), spec   # bf16 steps ran the persistent decode kernel
        for r in range(1, ws):                              # identical on every rank
            lgr, str_, _, _, chainr, _ = res[r]["model"][(str(dtype), spec)]
            assert np.array_equal(lg0, lgr), (spec, r)
            assert all(np.array_equal(a, b) for a, b in zip(st0, str_)), (spec, r)
            assert all(np.array_equal(a, b) for a, b in zip(chain0, chainr)), (spec, r)
        for a, c in zip(st0, chain0):                      # fused == chain up to accumulation order
            assert np.abs(a - c).max() <= 2e-2 * np.abs(c).max(), spec
        assert graph_ok, spec                              # graph replay == eager, bitwise
        # host-side count, as the reference's CommCounter: 2 per prefill (x2), 2 per eager step (3),
        # 2 per graph warm-up step (3) and 2 for the captured step; replays are not counted
        assert count == 2 * 2 + 2 * 3 + 2 * 3 + 2, count
        lm = O.OracleLM(O.Cfg(cfg.d_model, cfg.n_layer, cfg.vocab_size, dt_rank=cfg.dt_rank),
                        O.state_dict_numpy(sd), world_size=ws, spec=spec)
        ref, _ = lm.prefill(ids)
        if dtype_name == "float32":
            tol = {"fp32": 2e-4, "fp16": 2e-3}.get(spec, 2e-2)
            np.testing.assert_allclose(lg0, ref, atol=tol, rtol=1e-3)
            assert np.array_equal(lg0.argmax(-1), ref.argmax(-1)) or spec != "fp32"  # greedy tokens identical
        else:
            met = O.quant_metrics(ref, lg0)
            assert met["kl"].mean() <= 2e-3 and met["top1"].mean() >= 0.95, (spec, met)


# ------------------------------------------------------------------ per-tensor-scale variants in the model
@pytest.mark.parametrize("ws", WS_LIST)
def test_tp_model_with_per_tensor_scale_variants(ws):
    """int8_gather / int8_sum / int8_legacy sites (kernels over peer memory) mixed with
    per-row sites: the same logits on every rank, close to the oracle's TP emulation with
    the same map (prefill and one cached step), and the reference's accounting (int8_sum
    and int8_legacy count two collectives per call)."""
    if _ngpu() < ws:
        pytest.skip(f"needs {ws} GPUs")
    from mamba_tp_lite_b200.checkpoint import random_init_state_dict
    from mamba_tp_lite_b200.config import MambaConfig
    from mamba_tp_lite_b200.tp_utils import build_spec
    from oracle import mamba_oracle as O

    res = suite(ws)
    lg0, st0, count = res[0]["variants"]
    for r in range(1, ws):
        assert np.array_equal(res[r]["variants"][0], lg0) and np.array_equal(res[r]["variants"][1], st0), r
    assert count == 2 * (1 + 2)  # layer 0 per call (prefill, step): x_proj int8 1, out_proj int8_sum 2
    cfg = MambaConfig(d_model=256, n_layer=3, vocab_size=1000, dt_rank=16)
    sd = random_init_state_dict(cfg, seed=12, dtype=torch.float32)
    vspec = build_spec({"default": "int8", "overrides": {"0:out_proj": "int8_sum", "1:x_proj": "int8_gather",
                                                         "2:out_proj": "int8_legacy", "2:x_proj": "int8_sum",
                                                         "1:out_proj": "fp16"}}, cfg.n_layer)
    ids = torch.randint(0, cfg.vocab_size, (2, 72), generator=torch.Generator().manual_seed(4)).numpy()
    lm = O.OracleLM(O.Cfg(cfg.d_model, cfg.n_layer, cfg.vocab_size, dt_rank=cfg.dt_rank), O.state_dict_numpy(sd),
                    world_size=ws, spec=vspec)
    ref, _ = lm.prefill(ids)
    met = O.quant_metrics(ref, lg0)
    assert met["kl"].mean() <= 2e-3 and met["top1"].mean() >= 0.95, met


# ------------------------------------------------------------------ vocabulary-parallel lm_head
@pytest.mark.parametrize("ws", WS_LIST)
def test_vocab_parallel_lm_head_equals_replicated(ws):
    """Each rank computes V / ws logits columns and the ranks exchange them over peer
    memory: prefill logits (tensor-core and CUDA-core paths), step logits (GEMV path)
    and graphed greedy tokens are bit-identical to the replicated lm_head on every rank."""
    if _ngpu() < ws:
        pytest.skip(f"needs {ws} GPUs")
    res = suite(ws)
    for dtype in ("torch.float32", "torch.bfloat16"):
        rep = res[0]["vocab"][(dtype, "0")]
        for r in range(ws):
            got, ref = res[r]["vocab"][(dtype, "256")], res[r]["vocab"][(dtype, "0")]
            assert got[:3] == ref[:3] == rep[:3], (dtype, r)
            assert np.array_equal(got[3], ref[3]) and np.array_equal(got[3], rep[3]), (dtype, r)


# ------------------------------------------------------------------ x_proj reduction in the GEMM epilogue
@pytest.mark.parametrize("ws", WS_LIST)
def test_xproj_epilogue_reduction_equals_kernel_pair(ws):
    """The x_proj GEMM that writes AllReduce #1's wire rows (int8 / fp32 / fp16 sites)
    into every rank's slots plus the finishing reduction give the bits of the GEMM into
    an fp32 partial followed by the reduction kernel, on every rank."""
    if _ngpu() < ws:
        pytest.skip(f"needs {ws} GPUs")
    res = suite(ws)
    ref = res[0]["xfused"]["0"]
    for r in range(ws):
        assert res[r]["xfused"]["1"] == res[r]["xfused"]["0"], r  # logits and this rank's SSM states
        assert res[r]["xfused"]["1"][0] == ref[0], r               # the same logits on every rank


# ------------------------------------------------------------------ protocols agree (out_proj epilogue, bf16 gather)
@pytest.mark.parametrize("ws", WS_LIST)
def test_two_shot_bf16_gather_equals_one_shot(ws):
    if _ngpu() < ws:
        pytest.skip(f"needs {ws} GPUs")
    res = suite(ws)
    for mode in (0, 1, 2):
        a = res[0]["proto"][("oneshot", mode)]
        assert res[0]["proto"][("twoshot", mode)] == a, mode
        assert res[0]["proto"][("capped", mode)] == a, mode  # 16 CTAs, low-register kernel: same bits
        for r in range(1, ws):
            for proto in ("oneshot", "twoshot", "capped"):
                assert res[r]["proto"][(proto, mode)][:2] == a[:2], (r, proto, mode)
        # sequence-parallel epilogue: the same normed bits on every rank, and each rank's
        # residual rows equal the full epilogue's on the rows it owns
        for r in range(ws):
            sp, full = res[r]["proto"][("sp", mode)], res[r]["proto"][("oneshot", mode)]
            assert sp[1] == a[1], (r, mode)
            assert sp[2] == full[2], (r, mode)


# ------------------------------------------------------------------ overlapped micro-batch prefill == serial prefill
@pytest.mark.parametrize("ws", WS_LIST)
def test_overlapped_prefill_bit_exact_vs_serial(ws):
    if _ngpu() < ws:
        pytest.skip(f"needs {ws} GPUs")
    res = suite(ws)
    for r in range(ws):
        a, b = res[r]["overlap"]["1"], res[r]["overlap"]["0"]
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
        for (c1, s1), (c2, s2) in zip(a[2], b[2]):
            assert np.array_equal(c1, c2) and np.array_equal(s1, s2)
        assert a[3] == b[3] == 2 * 2  # the reference's accounting: 2 sites, 2 prefills
        assert np.array_equal(res[0]["overlap"]["1"][0], a[0])


# ------------------------------------------------------------------ bounded wait: a peer that never arrives
def _timeout_worker(rank, init_file, q, ws):
    try:
        import torch.distributed as dist

        _init(rank, init_file, ws)
        from mamba_tp_lite_b200 import _lib as L
        from mamba_tp_lite_b200.tp_utils import Comm

        comm = Comm(None, rank, ws, 64, 64, max_rows=64, timeout_s=1.0)
        x = torch.ones(8, 64, device="cuda")
        y = torch.empty_like(x)
        status = 0
        if rank == 0:  # rank 1 never enters this reduction: nothing sets rank 0's flag
            L.call("mtp_allreduce", comm.ptr, 1, L.RED_FP32, L.ptr(x), L.ptr(y), 8, 64, L.stream_ptr())
            torch.cuda.synchronize()
            status = comm.status()
            comm.reset_status()
            # the context's device is still usable after the bounded wait expired
            z = (x * 2).sum().item()
            assert z == 2 * 8 * 64
        dist.barrier()
        comm.destroy()
        q.put((rank, status))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, f"{type(e).__name__}: {e}"))


@needs(2)
def test_reduction_with_absent_peer_times_out_with_status():
    from mamba_tp_lite_b200 import _lib as L

    res = _spawn(_timeout_worker, 2)
    assert res[0] == L.MTP_ERR_TIMEOUT
    assert res[1] == 0


# ------------------------------------------------------------------ persistent decode: a peer that never steps
def _decode_timeout_worker(rank, init_file, q, ws):
    try:
        import time

        import torch.distributed as dist

        os.environ["MTP_COMM_TIMEOUT_S"] = "1"
        _init(rank, init_file, ws)
        from mamba_tp_lite_b200.checkpoint import random_init_state_dict
        from mamba_tp_lite_b200.config import MambaConfig
        from mamba_tp_lite_b200.tp_model import TPMambaLM
        from mamba_tp_lite_b200.tp_utils import get_comm

        cfg = MambaConfig(d_model=256, n_layer=2, vocab_size=512, dt_rank=16)
        sd = random_init_state_dict(cfg, seed=5, dtype=torch.bfloat16)
        m = TPMambaLM.from_state_dict_shard(cfg, sd, rank, ws, dtype=torch.bfloat16, allreduce_dtype="int8",
                                            device="cuda")
        ids = torch.randint(0, cfg.vocab_size, (2, 16), generator=torch.Generator().manual_seed(6)).cuda()
        _, cache = m.prefill(ids)  # both ranks: creates the comm context
        m.prepare_step(cache, 2)
        torch.cuda.synchronize()
        dist.barrier()
        result = (0, 0, 0.0)
        if rank == 0:  # rank 1 never steps: rank 0's AllReduce #1 wait must expire
            comm = get_comm(None, rank, ws, cfg.dt_rank + 2 * cfg.d_state, cfg.d_model)
            t0 = time.time()
            m.step(torch.zeros(2, 1, dtype=torch.long, device="cuda"), cache)
            torch.cuda.synchronize()
            result = (m._mtp_decode.status(), comm.status(), time.time() - t0)
            assert (torch.ones(8, device="cuda") * 2).sum().item() == 16  # context still usable
        # recovery: both ranks reset the decode plan and the comm context, then meet
        dist.barrier()
        comm = get_comm(None, rank, ws, cfg.dt_rank + 2 * cfg.d_state, cfg.d_model)
        m._mtp_decode.reset()
        comm.reset_state()
        dist.barrier()
        # a decode step (persistent kernel, peer reductions) and a plain reduction now succeed
        _, cache = m.prefill(ids)
        step = m.step(torch.zeros(2, 1, dtype=torch.long, device="cuda"), cache).float().cpu().numpy()
        from mamba_tp_lite_b200 import _lib as L
        x = torch.full((64, 64), float(rank + 1), device="cuda")
        y = torch.empty_like(x)
        L.call("mtp_allreduce", comm.ptr, 1, L.RED_FP32, L.ptr(x), L.ptr(y), 64, 64, L.stream_ptr())
        torch.cuda.synchronize()
        after = (m._mtp_decode.status(), comm.status(), float(y[0, 0]), step)
        q.put((rank, (result, after)))
        _finish()
    except Exception as e:
        q.put((rank, f"{type(e).__name__}: {e}"))


@needs(2)
def test_decode_kernel_with_absent_peer_times_out_with_status():
    from mamba_tp_lite_b200 import _lib as L

    res = _spawn(_decode_timeout_worker, 2)
    plan_status, comm_status, elapsed = res[0][0]
    assert plan_status == L.MTP_ERR_TIMEOUT and comm_status == L.MTP_ERR_TIMEOUT
    assert 0.5 < elapsed < 30
    assert res[1][0] == (0, 0, 0.0)
    # after mtp_decode_reset + mtp_comm_reset_state on every rank: clean statuses, the
    # reduction sums both ranks, and the decode step is identical on both ranks
    for r in (0, 1):
        p_st, c_st, red, _ = res[r][1]
        assert p_st == 0 and c_st == 0 and red == 3.0, (r, res[r][1][:3])
    assert np.array_equal(res[0][1][3], res[1][1][3])
