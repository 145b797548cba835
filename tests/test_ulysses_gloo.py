"""CPU, world_size 2 (gloo): the Ulysses sequence<->head all-to-all layout used around
attention by the multi-GPU DiT step."""
import itertools
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _host_permute(dst, src, chunk, dims, ss, ds):
    """qf2_copy_chunks restated through byte views on the host (gloo ranks have no GPU)."""
    def flat(t):
        n = t.untyped_storage().nbytes() // t.element_size()
        return torch.as_strided(t, (n,), (1,), 0).view(torch.uint8), t.storage_offset() * t.element_size()

    s8, bs = flat(src)
    d8, bd = flat(dst)
    for idx in itertools.product(*[range(n) for n in dims]):
        so = bs + sum(i * st for i, st in zip(idx, ss))
        do = bd + sum(i * st for i, st in zip(idx, ds))
        d8[do:do + chunk].copy_(s8[so:so + chunk])


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from quantfun2_b200.dit import SeqParallel, ulysses_attention

        g = torch.Generator().manual_seed(0)
        B, L, H, D = 2, 12, 4, 8
        full = [torch.randn(B, L, H, D, generator=g) for _ in range(3)]
        Ls = L // world
        local = [t[:, rank * Ls:(rank + 1) * Ls].contiguous() for t in full]
        sp = SeqParallel(dist.group.WORLD)
        heads = sp.seq_to_heads(local[0])
        # rank r holds every token for heads [r*H/P, (r+1)*H/P)
        ok1 = torch.equal(heads, full[0][:, :, rank * (H // world):(rank + 1) * (H // world)])
        ok2 = torch.equal(sp.heads_to_seq(heads), local[0])
        attn = lambda a, b, c: torch.nn.functional.scaled_dot_product_attention(  # noqa: E731
            a.transpose(1, 2), b.transpose(1, 2), c.transpose(1, 2)).transpose(1, 2)
        out = ulysses_attention(*local, sp, attn_fn=attn)
        ref = attn(*full)[:, rank * Ls:(rank + 1) * Ls]
        ok3 = torch.allclose(out, ref, atol=1e-6)
        # packed form: one exchange for q, k, v together, one for the output (B = 2 and 1)
        ok4 = True
        for bsz in (2, 1):
            qkv3 = torch.stack([t[:bsz] for t in local], dim=2).contiguous()  # [B, Ls, 3, H, D]
            dst = torch.full((bsz, Ls, H, D + 8), float("nan"))[..., :D]  # strided output rows

            def attn_o(a, b, c, o):
                o.copy_(attn(a, b, c))

            sp.attention_packed(qkv3, dst, attn_fn=attn_o, permute=_host_permute)
            ref_b = attn(*[t[:bsz] for t in full])[:, rank * Ls:(rank + 1) * Ls]
            ok4 = ok4 and torch.allclose(dst, ref_b, atol=1e-6)
        q.put((rank, ok1, ok2, ok3 and ok4))
    finally:
        dist.destroy_process_group()


def test_ulysses_all_to_all_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r[1] and r[2] and r[3] for r in res), res
