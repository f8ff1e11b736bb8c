"""Ulysses all-to-all layout, restated with numpy -- TEST INFRASTRUCTURE ONLY.

Follows comfyui_nodes/minimax-h3-sp/minimax_sp/sp_forward.py of the reference:
  SPContext splits / start / stop        :140-155
  forward pack + exchange (+no unpack)   :158-166, :179-188
  inverse exchange + unpack              :169-176, :191-198
  head-group pack of the overlap         :222-224
and the NCCL start-up known-answer test of sp_group.py:107-124.
The exchange of all ranks is simulated in one process: `sends[r]` is what rank
r hands to all_to_all_single and the function returns what every rank receives.
Pure data movement, so every comparison against it is bit-exact.
"""
import numpy as np


def splits(seq_len, world):
    """Rows per rank: base + 1 for the first `rem` ranks (sp_forward.py:148-149)."""
    base, rem = divmod(seq_len, world)
    return [base + (1 if r < rem else 0) for r in range(world)]


def starts(seq_len, world):
    sp = splits(seq_len, world)
    return [sum(sp[:r]) for r in range(world)]


def pack_fwd(t, world):
    """[s_local, H, Dh] -> send [P, s_local, (H/P)*Dh]  (sp_forward.py:185)."""
    s_local, heads, dim = t.shape
    hp = heads // world
    return np.ascontiguousarray(t.reshape(s_local, world, hp * dim).transpose(1, 0, 2))


def pack_group(t, world, groups, g):
    """Head group g of every destination's heads: [s_local, H, Dh] -> send
    [P, s_local, hc*Dh], hc = H/P/groups (prep() of sp_attention_overlap,
    sp_forward.py:222-224)."""
    s_local, heads, dim = t.shape
    w = heads // world // groups * dim
    return np.ascontiguousarray(t.reshape(s_local, world, groups, w)[:, :, g].transpose(1, 0, 2))


def a2a_fwd(ts, world):
    """All ranks' [s_local_r, H, Dh] -> every rank j's [S, H/P, Dh] (sp_forward.py:179-188).

    all_to_all_single sends block j of rank r's packed buffer to rank j, and rank
    j stores the blocks in source-rank order, which is sequence order."""
    heads, dim = ts[0].shape[1], ts[0].shape[2]
    hp = heads // world
    sends = [pack_fwd(t, world) for t in ts]
    return [np.concatenate([sends[r][j] for r in range(world)], axis=0).reshape(-1, hp, dim)
            for j in range(world)]


def a2a_inv(outs, world):
    """Every rank j's attention output [S, (H/P)*Dh] (contiguous per destination)
    -> every rank r's [s_local_r, H*Dh] (sp_forward.py:191-198)."""
    seq_len = outs[0].shape[0]
    chunk = outs[0].shape[1]
    sp, st = splits(seq_len, world), starts(seq_len, world)
    res = []
    for r in range(world):
        recv = np.stack([outs[j][st[r]:st[r] + sp[r]] for j in range(world)], axis=0)  # [P, s_loc, c]
        res.append(np.ascontiguousarray(recv.transpose(1, 0, 2)).reshape(sp[r], world * chunk))
    return res


def unpack_inv(recv, world):
    """[P, s_local, c] -> [s_local, P*c]  (the .transpose(0,1).reshape of sp_forward.py:198)."""
    p, s_local, c = recv.shape
    assert p == world
    return np.ascontiguousarray(recv.transpose(1, 0, 2)).reshape(s_local, p * c)


def startup_probe_expected(world, rank):
    """Known answers of sp_group.py:107-124: all_reduce of rank+1 sums to P(P+1)/2, and
    all_to_all_single of arange(P) + rank*P returns arange(P)*P + rank."""
    return world * (world + 1) / 2, np.arange(world, dtype=np.int64) * world + rank


def startup_probe_sources(world):
    return [np.arange(world, dtype=np.int64) + r * world for r in range(world)]
