"""Sequence parallelism on 2 GPUs (skipped with fewer): every rank runs the block on its token shard with
the in-place NCCL all-gather of the new chunk's K/V, and must reproduce the single-GPU block on the same
inputs (its rows of the output, and the whole destination chunk)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    from datetime import timedelta
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    import torch.distributed as dist
    import lbw_b200.block as B
    import lbw_b200.sp as sp
    from oracle.inputs import BlockCase, make_case
    try:
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
        case = BlockCase(dim=256, ffn=512, grid=(3, 4, 8), n_lead=2, text_len=32, start_frame=6, seed=41)
        p, inp = make_case(case)
        blk = B.CausalWanAttentionBlock(case.dim, case.ffn, case.heads, qk_norm=True, cross_attn_norm=True, ffn_mx=True)
        sd = blk.state_dict()
        for k, v in p.items():
            sd[k] = v.to(sd[k].dtype)
        blk.load_state_dict(sd)
        blk = blk.to(dev)
        C, H, Lq = case.dim, case.heads, case.lq
        bf = torch.bfloat16

        def run(x, film):
            ks = [k.unsqueeze(0).to(dev) for k in inp["k_lead"]] + [torch.zeros(1, Lq, H, 128, dtype=bf, device=dev)]
            vs = [v.unsqueeze(0).to(dev) for v in inp["v_lead"]] + [torch.zeros(1, Lq, H, 128, dtype=bf, device=dev)]
            cc = {"k": torch.zeros(1, case.text_len, H, 128, dtype=bf, device=dev),
                  "v": torch.zeros(1, case.text_len, H, 128, dtype=bf, device=dev), "is_init": torch.zeros(1, device=dev)}
            f, h, w = case.grid
            out = blk(x.unsqueeze(0).to(dev), inp["e0"].view(1, 1, 6, C).to(dev), grid_ints=[case.grid],
                      context=inp["context"].unsqueeze(0).to(dev), crossattn_cache=cc,
                      current_start=case.start_frame * h * w, frame_seqlen=h * w, kv_chunks=(ks, vs),
                      dit_cond_dict={"cam_film": (film[0].unsqueeze(0).to(dev), film[1].unsqueeze(0).to(dev))})
            torch.cuda.synchronize()
            return out[0].float().cpu(), ks[-1].cpu(), vs[-1].cpu()

        sp.set_group(None, enable=False)
        full, k_full, v_full = run(inp["x"], inp["film"])
        sp.set_group(None, enable=True)
        a, b = sp.shard_range(Lq)
        ok = True
        for _ in range(2):   # the second forward reuses the exchange buffers (next epoch)
            mine, k_sp, v_sp = run(inp["x"][a:b], (inp["film"][0][a:b], inp["film"][1][a:b]))
            rel = float((mine - full[a:b]).norm() / full[a:b].norm())
            ok = ok and rel < 1e-3 and torch.equal(k_sp, k_full) and torch.equal(v_sp, v_full)
        q.put((rank, "ok" if ok else f"mismatch rel {rel:.3e} k {torch.equal(k_sp, k_full)} v {torch.equal(v_sp, v_full)}"))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_sequence_parallel_block_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


def _gather_worker(rank, world, port, q):
    import sys
    from datetime import timedelta
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.load_package()
    import torch.distributed as dist
    import lbw_b200.sp as sp
    try:
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
        sp.set_group(None, enable=True)
        rows, cols, ld = 300, 384, 512            # ragged row count, padded row stride
        ok = True
        for it in range(4):
            k = torch.full((world * rows, ld), -1.0, dtype=torch.bfloat16, device=dev)
            v = torch.full((world * rows, ld), -1.0, dtype=torch.bfloat16, device=dev)
            ri = torch.arange(rows, device=dev).view(rows, 1) % 7
            ci = torch.arange(cols, device=dev).view(1, cols) % 5
            want_k = torch.cat([(r * 10 + it) + ri * 0.5 + ci * 0.25 for r in range(world)]).to(torch.bfloat16)
            want_v = -want_k
            k[rank * rows:(rank + 1) * rows, :cols] = want_k[rank * rows:(rank + 1) * rows]
            v[rank * rows:(rank + 1) * rows, :cols] = want_v[rank * rows:(rank + 1) * rows]
            sp.gather_kv_inplace(k[:, :cols], v[:, :cols], rows)
            torch.cuda.synchronize()
            ok = ok and torch.equal(k[:, :cols], want_k) and torch.equal(v[:, :cols], want_v)
            ok = ok and bool((k[:, cols:] == -1).all()) and bool((v[:, cols:] == -1).all())   # padding untouched
        sp.close_peers()
        q.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_peer_kv_gather_two_gpus():
    """The copy-engine K/V exchange over four epochs (buffer reuse), ragged rows and a padded row stride."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
