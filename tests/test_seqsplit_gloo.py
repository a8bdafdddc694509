"""CPU, world size 2 (gloo): the sequence-split protocol of
zoomkv_revision_b200.seqsplit (score exchange, global selection, per-rank
attention over owned pages, log-sum-exp merge) with the oracle as the
compute backend; the merged result must equal the single-device oracle page
decode (selection exact, output within the attention tolerance)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

G, D = 4, 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_data(seed, R, n_c, n_near):
    """Full synthetic layer (numpy): K/V with outlier key channels."""
    rng = np.random.default_rng(seed)
    T = n_c * 16
    k = rng.standard_normal((R, T + n_near, D)).astype(np.float32)
    k[:, :, rng.choice(D, 4, replace=False)] *= 10
    v = rng.standard_normal((R, T + n_near, D)).astype(np.float32)
    q = rng.standard_normal((R, G, D)).astype(np.float32)
    kb, vb, qb = O.f32_to_bf16(k), O.f32_to_bf16(v), O.f32_to_bf16(q)
    mn, mx, ce, pk = O.kivi_encode_chunks(kb[:, :T])
    vc, vm = O.vquant_tokens(vb[:, :T])
    return dict(q=qb, mn=mn, mx=mx, pk=pk, vc=vc, vm=vm, near_k=kb[:, T:], near_v=vb[:, T:], n_c=n_c,
                n_near=n_near)


class Layer:
    """Rank-local layer for the oracle backend: pages [lo, hi) of the data."""

    def __init__(self, data, lo, hi, bs, H):
        self.d, self.lo, self.hi = data, lo, hi
        self.tensors = (torch.empty(bs, H, 0, D),)


class OracleBackend:
    def raw_q(self, q, heads):
        qf = O.bf16_to_f32(q.view(torch.int16).numpy().view(np.uint16)).reshape(-1, G, D)
        acc = np.zeros((qf.shape[0], D), np.float32)
        for g in range(G):
            acc = (acc + qf[:, g]).astype(np.float32)
        rq = O.f32_to_bf16(acc / np.float32(G))
        return torch.from_numpy(rq.view(np.int16)).view(torch.bfloat16).reshape(q.shape[0], heads, D)

    def local_scores(self, raw_q, layer, n_loc, local, out):
        if n_loc > 0:
            d, lo = layer.d, layer.lo
            rq = raw_q.view(torch.int16).numpy().view(np.uint16).reshape(-1, D)
            sc = O.quest_score(rq, np.ascontiguousarray(d["mn"][:, lo:lo + n_loc]),
                               np.ascontiguousarray(d["mx"][:, lo:lo + n_loc]), None, n_loc)
            out[:, :, :n_loc] = torch.from_numpy(sc).view(out.shape[0], out.shape[1], n_loc)
        return out

    def global_topk(self, scores, nk, out):
        R = scores.shape[0] * scores.shape[1]
        sel = O.topk_f32(scores.reshape(R, -1).numpy(), nk)
        out.copy_(torch.from_numpy(sel).view(out.shape))
        return out

    def attend(self, q, layer, sel, lo, hi, n_sink, near_start, n_near, out_f32, lse, status):
        d = layer.d
        qf = O.bf16_to_f32(q.view(torch.int16).numpy().view(np.uint16)).reshape(-1, G, D)
        s = sel.reshape(qf.shape[0], -1).numpy()
        for r in range(qf.shape[0]):
            ks, vs = [], []
            for c in s[r]:
                if lo <= c < hi:
                    ks.append(O.kivi_dequant_chunk(d["pk"][r, c], d["mn"][r, c], d["mx"][r, c]))
                    vs.append(O.vdequant_tokens(d["vc"][r, 16 * c:16 * c + 16], d["vm"][r, 16 * c:16 * c + 16]))
            if n_near:
                ks.append(d["near_k"][r, near_start:near_start + n_near])
                vs.append(d["near_v"][r, near_start:near_start + n_near])
            if ks:
                o, l = O.attn_dense(qf[r], O.bf16_to_f32(np.concatenate(ks)), O.bf16_to_f32(np.concatenate(vs)),
                                    1 / np.sqrt(D))
            else:
                o, l = np.zeros((G, D), np.float32), np.full(G, -np.inf, np.float32)
            out_f32.view(-1, G, D)[r] = torch.from_numpy(o)
            lse.view(-1, G)[r] = torch.from_numpy(l)
        return out_f32

    def merge(self, parts, lses, out):
        p, l = parts.numpy().astype(np.float64), lses.numpy().astype(np.float64)
        m = l.max(axis=0)
        w = np.where(np.isfinite(l), np.exp(l - m), 0.0)
        o = (w[..., None] * p).sum(0) / w.sum(0)[..., None]
        out.copy_(torch.from_numpy(O.f32_to_bf16(o.astype(np.float32)).view(np.int16)).view(torch.bfloat16))
        return out


def _rank_main(rank, world, port, case, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from zoomkv_revision_b200 import seqsplit as S
        bs, H, n_c, nk, n_near, seed = case
        data = make_data(seed, bs * H, n_c, n_near)
        lo, hi, per = S.split_range(n_c, world, rank)
        bufs = S.SplitBuffers.alloc(bs, H, G, per, nk, world, "cpu")
        q = torch.from_numpy(data["q"].view(np.int16)).view(torch.bfloat16).reshape(bs, 1, H * G, D)
        out, sel = S.decode_step(q, Layer(data, lo, hi, bs, H), n_c, nk, bufs, rank=rank, world=world,
                                 n_near=n_near, backend=OracleBackend())
        np.savez(os.path.join(result_dir, f"r{rank}.npz"), out=out.view(torch.int16).numpy(), sel=sel.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(1, 2, 37, 9, 24, 0), (2, 1, 64, 16, 16, 1), (1, 2, 40, 40, 8, 2)])
def test_seqsplit_world2_matches_single_device(tmp_path, case):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), case, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    bs, H, n_c, nk, n_near, seed = case
    data = make_data(seed, bs * H, n_c, n_near)
    vct, vmt = O.page_layout_values(data["vc"], data["vm"])
    ro, _, rsel = O.page_decode(data["q"], data["mn"], data["mx"], None, data["pk"], vct, vmt, data["near_k"],
                                data["near_v"], n_c, nk, n_near, 1 / np.sqrt(D))
    res = [np.load(os.path.join(tmp_path, f"r{r}.npz")) for r in range(world)]
    for r in res:   # every rank holds the same merged result and selection
        assert np.array_equal(r["sel"].reshape(bs * H, nk), rsel)
        assert np.array_equal(r["out"], res[0]["out"])
    out = O.bf16_to_f32(res[0]["out"].view(np.uint16)).reshape(bs * H, G, D)
    ref = O.bf16_to_f32(ro)
    err = np.abs(out - ref)
    assert err.max() <= 2e-2 and err.mean() / np.abs(ref).mean() <= 1e-2, (err.max(), err.mean())


@pytest.mark.parametrize("world,rows,n_c", [(1, 8, 8184), (2, 8, 8184), (3, 2, 1001), (8, 8, 8184), (8, 64, 2040)])
def test_peer_buffer_layout(world, rows, n_c):
    """The shared buffer of the peer-memory transport: the flag arrays, the
    epoch and the CTA counter fit the header; regions are 256-byte aligned and
    disjoint; every rank's score slice and partial slots land inside their
    region and do not overlap another rank's."""
    from zoomkv_revision_b200 import seqsplit as S
    G, P = 4, 4
    per = S.split_range(n_c, world, 0)[2]
    lay = S.peer_layout(rows, G, per, world, P)
    assert S._FLAGS_A + 4 * 8 <= S._FLAGS_B and S._FLAGS_B + 4 * 8 <= S._EPOCH and S._DONE + 4 <= S._HEADER
    assert all(lay[k] % 256 == 0 for k in ("row", "parts", "lses", "total"))
    assert lay["row"] + rows * world * per * 4 <= lay["parts"]
    assert lay["parts"] + world * P * rows * G * 128 * 4 <= lay["lses"]
    assert lay["lses"] + world * P * rows * G * 4 <= lay["total"]
    covered = set()
    for r in range(world):
        lo, hi, _ = S.split_range(n_c, world, r)
        assert 0 <= hi - lo <= per
        # score slice of rank r: columns [r*per, r*per + n_loc) of every row
        cols = set(range(r * per, r * per + (hi - lo)))
        assert not (cols & covered)
        covered |= cols
    assert covered == set(range(n_c))  # every chunk has exactly one owner; columns past n_c stay -inf
