"""CPU, world_size 2/3/4 over gloo: the Ulysses exchanges and the K/V
all-gather of minixmax_h3_b200.ulysses reproduce the reference's layouts
(ops/ulysses.py, runtime/dist.py) bit-for-bit, the ring scheme
(ops/fa_h3.py:141-218) with the oracle's attention and LSE merge plugged in
matches attention over every rank's keys, and the failures a rank can cause
(it dies, it stalls past the process group's timeout, it sends a message of
the wrong size) reach the others as errors, not hangs or aborts."""
from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, ws: int, port: int, mode: str, results) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        short = mode in ("slow_peer", "bad_size")  # these wait for the process group's timeout
        dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=3 if short else 20))
        from minixmax_h3_b200 import dist as hdist
        from minixmax_h3_b200 import ulysses as U
        from oracle import h3_oracle as O

        hdist.set_state(rank, ws, group=dist.group.WORLD, backend="gloo")
        check = mode == "bad_size"  # exchanges confirm the message shapes first
        s, h, d = 6 * ws, 2 * ws, 4
        full = torch.arange(s * h * d, dtype=torch.float32).reshape(s, h, d)
        s0, s1 = U.split_range(s)
        assert (s0, s1) == O.split_range(s, ws, rank)
        local = full[s0:s1].contiguous()
        if mode == "exchange":
            got = U.all_to_all_heads(local, gather_seq=True)
            assert torch.equal(got, O.seq_to_head_local(full, ws, rank))
            back = U.all_to_all_heads(got, gather_seq=False)
            assert torch.equal(back, local)
            qkv_full = torch.randn(s, 3, h, d, generator=torch.Generator().manual_seed(1))
            tq, tk, tv = U.all_to_all_qkv(qkv_full[s0:s1].reshape(s1 - s0, -1).contiguous(), h, d)
            for t, part in ((tq, 0), (tk, 1), (tv, 2)):
                assert torch.equal(t, O.seq_to_head_local(qkv_full[:, part], ws, rank))
            # all-gather of K and V (runtime/dist.py:291-312): full tensors in rank order
            kf = torch.randn(s, h, d, generator=torch.Generator().manual_seed(2))
            vf = torch.randn(s, h, d, generator=torch.Generator().manual_seed(3))
            kg, vg = U.all_gather_kv(kf[s0:s1].contiguous(), vf[s0:s1].contiguous())
            assert torch.equal(kg, kf) and torch.equal(vg, vf)
            segs = [(0, 5, 1), (5, s, 0)]
            assert U.clip_mod_segments(segs, s0, s1) == O.clip_mod_segments(segs, s0, s1)
            results.put((rank, "ok"))
        elif mode == "ring":
            g = torch.Generator().manual_seed(7)
            qf, kf, vf = (torch.randn(s, h, 16, generator=g).to(torch.bfloat16) for _ in range(3))

            def attn(q_, k_, v_, sc, o_, lse_):
                o, lse = O.attention_lse_fp32(q_, k_, v_, sc)
                o_.copy_(o.to(torch.bfloat16))
                lse_.copy_(lse)

            def merge(acc, acc_lse, blk, blk_lse, first, out=None, amax_out=None):
                if first:
                    acc.copy_(blk.float())
                    acc_lse.copy_(blk_lse)
                else:
                    o, lse = O.merge_lse(acc, acc_lse, blk, blk_lse)
                    acc.copy_(o)
                    acc_lse.copy_(lse)
                if out is not None:
                    out.copy_(acc.to(torch.bfloat16))

            got = U.ring_attention(qf[s0:s1], kf[s0:s1], vf[s0:s1], attention_fn=attn, merge_fn=merge)
            want, _ = O.attention_lse_fp32(qf[s0:s1], kf, vf)
            err = (got.float() - want).abs().max().item()
            results.put((rank, "ok" if err < 1e-2 else f"ring err {err}"))
        elif mode == "dead_peer":
            U.all_to_all_heads(local, gather_seq=True, check_shapes=check)  # a healthy step: connections are up
            if rank == ws - 1:
                results.put((rank, "exited"))
                results.close()
                results.join_thread()  # flush before the hard exit
                os._exit(0)  # leaves between steps, nothing in flight
            try:
                U.all_to_all_heads(local, gather_seq=True)
                results.put((rank, "no error"))
            except Exception as e:  # noqa: BLE001 - any transport error is the expected outcome
                results.put((rank, f"error:{type(e).__name__}"))
        elif mode == "bnsd_entries":
            # the reference's BNSD sequence-parallel entries, with the oracle's
            # fp32 attention and LSE merge standing in for the two kernels
            from minixmax_h3_b200 import attention as A
            from minixmax_h3_b200 import ops

            def fake_attention(q_, k_, v_, *, scale=None, out=None, lse=None, amax_out=None):
                o, l_ = O.attention_lse_fp32(q_, k_, v_, scale)
                out = torch.empty(q_.shape, dtype=torch.bfloat16) if out is None else out
                out.copy_(o.to(torch.bfloat16))
                if lse is not None:
                    lse.copy_(l_)
                return out

            def fake_merge(acc, acc_lse, blk, blk_lse, *, first, out=None, amax_out=None):
                if first:
                    acc.copy_(blk.float())
                    acc_lse.copy_(blk_lse)
                else:
                    o, l_ = O.merge_lse(acc, acc_lse, blk, blk_lse)
                    acc.copy_(o)
                    acc_lse.copy_(l_)
                if out is not None:
                    out.copy_(acc.to(torch.bfloat16))

            ops.attention, ops.attention_merge_lse = fake_attention, fake_merge
            g = torch.Generator().manual_seed(11)
            qf, kf, vf = (torch.randn(s, h, 16, generator=g).to(torch.bfloat16) for _ in range(3))
            want, _ = O.attention_lse_fp32(qf[s0:s1], kf, vf)  # local queries, every key
            want = want.permute(1, 0, 2).unsqueeze(0)  # [1, H, S_local, D]

            def bnsd(t):
                return t[s0:s1].permute(1, 0, 2).unsqueeze(0).contiguous()

            qb, kb, vb = bnsd(qf), bnsd(kf), bnsd(vf)
            errs = {
                "gather_fa_bnsd": A.gather_fa_bnsd(qb, kb, vb),
                "sp_gather_fa": A.sp_gather_fa(qb[0], kb[0], vb[0]).unsqueeze(0),
            }
            errs["ring_attention_bnsd"] = A.ring_attention_bnsd(qb, kb, vb)
            bad = {n: (o.shape, (o.float() - want).abs().max().item()) for n, o in errs.items()
                   if o.shape != want.shape or (o.float() - want).abs().max().item() > 1e-2}
            results.put((rank, "ok" if not bad else f"bnsd {bad}"))
        elif mode in ("slow_peer", "bad_size"):
            import time

            U.all_to_all_heads(local, gather_seq=True, check_shapes=check)  # a healthy step: connections are up
            x = local
            if rank == ws - 1:
                if mode == "slow_peer":
                    time.sleep(8)  # past the others' 3 s timeout
                else:
                    x = local[:-1].contiguous()  # one token short: a wrong message size
            t0 = time.monotonic()
            try:
                U.all_to_all_heads(x, gather_seq=True, check_shapes=check)
                results.put((rank, "no error"))
            except Exception as e:  # noqa: BLE001 - any transport error is the expected outcome
                results.put((rank, f"error:{type(e).__name__}:{time.monotonic() - t0:.1f}:{str(e)[:80]}"))
            return  # the group is broken; leave without a collective teardown
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        results.put((rank, f"fail:{e!r}"))


def _run(ws: int, mode: str, timeout: float = 120.0) -> dict:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, mode, q)) for r in range(ws)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(ws):
            r, msg = q.get(timeout=timeout)
            out[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out


@pytest.mark.parametrize("ws", [2, 4])
def test_ulysses_exchanges_match_reference_layout(ws):
    res = _run(ws, "exchange")
    assert res == {r: "ok" for r in range(ws)}, res


@pytest.mark.parametrize("ws", [2, 3])
def test_ring_attention_matches_full_attention(ws):
    res = _run(ws, "ring")
    assert res == {r: "ok" for r in range(ws)}, res


@pytest.mark.parametrize("ws", [2, 3])
def test_bnsd_sequence_parallel_entries(ws):
    """gather_fa_bnsd, sp_gather_fa and ring_attention_bnsd (the
    reference's ops/gather_fa.py and ops/ring_attention.py entries): each
    rank's queries against every rank's keys, as attention over the full
    sequence."""
    res = _run(ws, "bnsd_entries")
    assert res == {r: "ok" for r in range(ws)}, res


def test_dead_peer_is_reported_not_hung():
    res = _run(2, "dead_peer")
    assert res[1] == "exited"
    assert res[0].startswith("error:"), res


def _error(msg: str) -> tuple[str, float, str]:
    _, kind, secs, text = msg.split(":", 3)
    return kind, float(secs), text


def test_slow_peer_times_out_cleanly():
    """A rank that stalls past the process group's timeout (3 s here): the
    waiting rank gets an error after about that long instead of hanging, and
    the late rank gets one as soon as it arrives."""
    res = _run(2, "slow_peer")
    assert res[0].startswith("error:") and res[1].startswith("error:"), res
    _, secs, _ = _error(res[0])
    assert 2.5 <= secs <= 10, res


def test_wrong_message_size_is_a_clean_error():
    """One rank sends a sequence slice one token short.  Unchecked, gloo would
    abort the receiving process; with check_shapes=True every rank raises
    the same RuntimeError before the exchange."""
    res = _run(2, "bad_size")
    for r in (0, 1):
        kind, secs, text = _error(res[r])
        assert kind == "RuntimeError" and "exchange mismatch" in text and secs < 2.5, res
