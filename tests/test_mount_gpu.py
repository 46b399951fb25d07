"""Fused dequant + scatter mount and the arena splice on the GPU, against the
reference goldens (core/graft_quant.py, DeviceArena::apply_swap_tensor) and the
CPU oracle.  Bytes must be bit-exact; seats outside the mount keep the fill."""

import numpy as np
import pytest

import oracle as O
from graftrepository_b200 import GrmB200Error, graft_mount, synth

pytestmark = pytest.mark.gpu
SENTINEL = 0x7F81  # a NaN bf16 pattern no dequant produces


def _u16(t):
    import torch
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("bits", [8, 6, 4, 3, 2])
def test_ref_format_golden(golden, bits):
    import torch

    g = golden("quant_g32.npz")
    x = g["x_f16"].view(np.float16)                      # [2, 3, 8, 96]
    # treat axis 0 as grafts, axis 1 as layers, (8 tokens x 96 values) per slice
    codes = torch.from_numpy(g[f"codes{bits}"].reshape(2, 3, -1)).cuda()
    scales = torch.from_numpy(g[f"scales{bits}"].reshape(2, 3, -1)).cuda()
    seats = np.array([5, 20], dtype=np.int64)
    m = graft_mount.ArenaMount(3, 40, 96, fill=SENTINEL)
    m.mount_ref(codes, scales, seats, tokens=8)
    got = _u16(m.arena)
    want = np.full((3, 40, 96), SENTINEL, np.uint16)
    deq = g[f"dequant_bf16_{bits}"].reshape(2, 3, 8, 96)
    want = O.mount_scatter(deq, seats, want)
    assert np.array_equal(got, want)
    assert x.shape == (2, 3, 8, 96)


@pytest.mark.parametrize("bits", [8, 6, 4])
def test_packed_format_matches_oracle(bits):
    import torch

    vals = synth.grafts(40 + bits, 3, 5, 128, 288)
    codes, scales = graft_mount.quantize_packed(vals.reshape(3, 5, -1), bits)
    seats = synth.seat_offsets(bits, 3, 128, 1000)
    m = graft_mount.ArenaMount(5, 1000, 288, fill=SENTINEL)
    m.mount_packed(torch.from_numpy(codes).cuda(),
                   torch.from_numpy(scales.view(np.uint16)).cuda(), seats, 128, bits)
    deq = O.dequant_packed(codes.reshape(-1), scales.view(np.uint16).reshape(-1), bits)
    want = O.mount_scatter(deq.reshape(3, 5, 128, 288), seats,
                           np.full((5, 1000, 288), SENTINEL, np.uint16))
    assert np.array_equal(_u16(m.arena), want)


def test_full_size_config5_int4_and_ref():
    """3 grafts x 62 layers x 2048 tokens x 288 values into arena [62, 8192, 288]."""
    import torch

    vals = synth.grafts(4)
    seats = synth.seat_offsets(4, 3, 2048, 8192)
    for bits in (4, 6, 8):
        codes, scales = graft_mount.quantize_packed(vals.reshape(3, 62, -1), bits)
        m = graft_mount.ArenaMount(62, 8192, 288, fill=SENTINEL)
        m.mount_packed(torch.from_numpy(codes).cuda(),
                       torch.from_numpy(scales.view(np.uint16)).cuda(), seats, 2048, bits)
        got = _u16(m.arena)
        deq = O.dequant_packed(codes.reshape(-1), scales.view(np.uint16).reshape(-1), bits)
        want = O.mount_scatter(deq.reshape(3, 62, 2048, 288), seats,
                               np.full((62, 8192, 288), SENTINEL, np.uint16))
        assert np.array_equal(got, want), bits
        del m
    # reference format (graft_quant group 32, fp32 scales) at full size
    c32, s32 = O.quant_ref(vals, 8)
    m = graft_mount.ArenaMount(62, 8192, 288, fill=SENTINEL)
    m.mount_ref(torch.from_numpy(c32.reshape(3, 62, -1)).cuda(),
                torch.from_numpy(s32.reshape(3, 62, -1)).cuda(), seats, tokens=2048)
    _, bf = O.dequant_ref(c32, s32)
    want = O.mount_scatter(bf.reshape(3, 62, 2048, 288), seats,
                           np.full((62, 8192, 288), SENTINEL, np.uint16))
    assert np.array_equal(_u16(m.arena), want)


def test_seat_overflow_is_rejected():
    import torch

    codes = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(32, dtype=torch.int16, device="cuda")
    arena = torch.zeros((1, 10, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(GrmB200Error):
        graft_mount.mount_packed(codes, scales, [5], arena, bits=8, layers=1, tokens=8, width=64)


def test_splice_golden(golden):
    import torch

    g = golden("splice.npz")
    i = 0
    while f"c{i}_params" in g:
        sink, width, old_mount = (int(v) for v in g[f"c{i}_params"])
        old = g[f"c{i}_old"]
        mnt = g[f"c{i}_mount"]
        outer, tin, inner = old.shape
        # pad rows to a 16-byte multiple: 10 uint16 -> 16 uint16
        pad = 16 - inner
        oldp = np.concatenate([old, np.zeros((outer, tin, pad), np.uint16)], axis=2)
        mntp = np.concatenate([mnt, np.zeros((outer, mnt.shape[1], pad), np.uint16)], axis=2)
        exp = g[f"c{i}_out"]
        out = torch.zeros((outer, exp.shape[1], 16), dtype=torch.int16, device="cuda")
        t_old = torch.from_numpy(oldp.view(np.int16)).cuda()
        t_m = torch.from_numpy(mntp.view(np.int16)).cuda() if mnt.shape[1] else None
        got_t = graft_mount.arena_splice(t_old, t_m, out, outer=outer, input_tokens=tin,
                                         mount_tokens=mnt.shape[1], row_bytes=32,
                                         sink_tokens=sink, old_mount_tokens=old_mount)
        assert got_t == exp.shape[1]
        got = out.cpu().numpy().view(np.uint16)[:, :, :inner]
        assert np.array_equal(got, exp), i
        i += 1


def _rope_dev(rows, dim):
    import torch

    c, s = graft_mount.rope_tables(rows, dim)
    return c, s, torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda()


@pytest.mark.parametrize("bits", [8, 6, 4, 0])
@pytest.mark.parametrize("W,offset,dim,pair_swap", [(288, 256, 32, False), (288, 256, 32, True),
                                                    (256, 0, 128, False), (192, 64, 64, True),
                                                    (288, 32, 64, False), (288, 96, 96, True)])
def test_rope_mount_matches_oracle(bits, W, offset, dim, pair_swap):
    """Dequant + scatter + re-RoPE of the positional columns at the arena seats
    in one kernel == oracle mount followed by orc_mount_rope, bit-exact
    (bits 0: the reference format)."""
    import torch

    G, L, T, S = 3, 4, 96, 700
    vals = synth.grafts(60 + bits + dim, G, L, T, W)
    seats = synth.seat_offsets(bits + W, G, T, S)
    c, s, dc, ds = _rope_dev(S, dim)
    rope = graft_mount.RopeSpec(dc, ds, offset, dim, pair_swap)
    m = graft_mount.ArenaMount(L, S, W, fill=SENTINEL)
    if bits:
        codes, scales = graft_mount.quantize_packed(vals.reshape(G, L, -1), bits)
        m.mount_packed(torch.from_numpy(codes).cuda(),
                       torch.from_numpy(scales.view(np.uint16)).cuda(), seats, T, bits,
                       rope=rope)
        deq = O.dequant_packed(codes.reshape(-1), scales.view(np.uint16).reshape(-1), bits)
    else:
        c32, s32 = O.quant_ref(vals, 8)
        m.mount_ref(torch.from_numpy(c32.reshape(G, L, -1)).cuda(),
                    torch.from_numpy(s32.reshape(G, L, -1)).cuda(), seats, T, rope=rope)
        _, deq = O.dequant_ref(c32, s32)
    want = O.mount_scatter(deq.reshape(G, L, T, W), seats,
                           np.full((L, S, W), SENTINEL, np.uint16))
    want = O.mount_rope(want, G, L, T, seats, c, s, offset, dim, pair_swap)
    assert np.array_equal(_u16(m.arena), want)


def test_rope_mount_full_size_config5_int4():
    """3 grafts x 62 layers x 2048 tokens x 288 values (k_pe 32 at column 256)
    re-RoPEd at arena seats up to 8192."""
    import torch

    vals = synth.grafts(4)
    seats = synth.seat_offsets(4, 3, 2048, 8192)
    c, s, dc, ds = _rope_dev(8192, 32)
    codes, scales = graft_mount.quantize_packed(vals.reshape(3, 62, -1), 4)
    m = graft_mount.ArenaMount(62, 8192, 288, fill=SENTINEL)
    m.mount_packed(torch.from_numpy(codes).cuda(), torch.from_numpy(scales.view(np.uint16)).cuda(),
                   seats, 2048, 4, rope=graft_mount.RopeSpec(dc, ds, 256, 32))
    deq = O.dequant_packed(codes.reshape(-1), scales.view(np.uint16).reshape(-1), 4)
    want = O.mount_scatter(deq.reshape(3, 62, 2048, 288), seats,
                           np.full((62, 8192, 288), SENTINEL, np.uint16))
    want = O.mount_rope(want, 3, 62, 2048, seats, c, s, 256, 32)
    assert np.array_equal(_u16(m.arena), want)


@pytest.mark.parametrize("offset,dim,rows", [(250, 32, 700), (256, 24, 700), (256, 32, 100)])
def test_rope_mount_rejects_bad_specs(offset, dim, rows):
    import torch

    codes = torch.zeros(8 * 288 // 2, dtype=torch.uint8, device="cuda")
    scales = torch.zeros(8 * 288 // 64, dtype=torch.int16, device="cuda")
    arena = torch.zeros((1, 700, 288), dtype=torch.bfloat16, device="cuda")
    c = torch.zeros((rows, dim), dtype=torch.float32, device="cuda")
    with pytest.raises(GrmB200Error):
        graft_mount.mount_packed(codes, scales, [200], arena, bits=4, layers=1, tokens=8,
                                 width=288, rope=graft_mount.RopeSpec(c, c, offset, dim))


@pytest.mark.parametrize("tag,names", [("mla8", ("c", "kpe")), ("mla4", ("c", "kpe")),
                                       ("gqa6", ("k",)), ("gqa3", ("k",))])
@pytest.mark.parametrize("with_rope", [False, True])
def test_packed_payloads_mount_like_unpack_kv_arrays(golden, tag, names, with_rope):
    """Payloads written by the reference's pack_kv_arrays, uploaded as stored
    and mounted by the fused kernel == the reference's unpack_kv_arrays
    output cast to bf16, rows [c | kpe] (MLA) or L*H slices (GQA), scattered
    to the seats; with rope, then re-RoPEd (oracle) at the seats."""
    from graftrepository_b200 import packed

    g = golden("packed_payload.npz")
    pre = f"{tag}__"
    pl = {k[len(pre):]: g[k] for k in g if k.startswith(pre)}
    shapes = {n: tuple(int(x) for x in pl[f"{n}_shape"]) for n in names}
    lead = shapes[names[0]][:-1]
    slices, tokens = int(np.prod(lead[:-1])), lead[-1]
    width = sum(shapes[n][-1] for n in names)
    # two nodes: the payload and a copy with its codes negated
    pl2 = dict(pl)
    for n in names:
        pl2[f"{n}_codes"] = (-pl[f"{n}_codes"].astype(np.int16)).clip(-128, 127).astype(np.int8)
    S = 3 * tokens + 5
    seats = np.array([tokens + 2, 0], dtype=np.int64)
    m = graft_mount.ArenaMount(slices, S, width, fill=SENTINEL)
    rope = None
    if with_rope:
        off, dim = (256, 32) if names == ("c", "kpe") else (0, width)
        c_tab, s_tab = graft_mount.rope_tables(S, dim)
        import torch
        rope = graft_mount.RopeSpec(torch.from_numpy(c_tab).cuda(), torch.from_numpy(s_tab).cuda(),
                                    off, dim, pair_swap=(tag == "mla4"))
    packed.mount_payloads(m, [pl, pl2], seats, names, rope=rope)
    vals = []
    for p in (pl, pl2):
        parts = []
        for n in names:
            _, bf = O.dequant_ref(p[f"{n}_codes"].reshape(-1), p[f"{n}_scales"].reshape(-1))
            parts.append(bf.reshape(slices, tokens, shapes[n][-1]))
        vals.append(np.concatenate(parts, axis=-1))
    want = O.mount_scatter(np.stack(vals), seats, np.full((slices, S, width), SENTINEL, np.uint16))
    if with_rope:
        want = O.mount_rope(want, 2, slices, tokens, seats, c_tab, s_tab, off, dim,
                            pair_swap=(tag == "mla4"))
    assert np.array_equal(_u16(m.arena), want)
    # node 1 of the payload is exactly the reference's own output
    if not with_rope:
        ref = np.concatenate([pl[f"expect_bf16_{n}"].reshape(slices, tokens, -1) for n in names],
                             axis=-1)
        assert np.array_equal(_u16(m.arena)[:, seats[0]:seats[0] + tokens], ref)
