"""The end-to-end leg of ``bench.py`` moves a step's inputs and outputs as one
copy per group of four layers: every layer's tensors are views of one packed
buffer.  Checked here on CPU tensors: the views keep their values and shapes,
start 256 bytes apart at least (the kernels read them with 16-byte vector
loads), and each group's range covers exactly its four layers' tensors."""
import torch

import bench

T = 8


def _step():
    s = bench.Step.__new__(bench.Step)           # no device: only the packing is exercised
    s.torch, s.dev, s.rank = torch, torch.device('cpu'), 0
    g = torch.Generator().manual_seed(3)
    r = lambda *shape: torch.randn(*shape, generator=g)  # noqa: E731
    s.attn = [dict(q_gate=r(T, 24, 512), key=r(T, 4, 256), value=r(T, 4, 256), out=torch.zeros(T, 24, 256))
              for _ in range(bench.LAYERS // 4)]
    s.delta = [dict(qkv=r(T, 10240), gate=r(T, 48, 128), alpha=r(T, 48), beta=r(T, 48), out=torch.zeros(T, 48, 128))
               for _ in range(3 * bench.LAYERS // 4)]
    return s


def test_packed_views_keep_values_and_alignment():
    s = _step()
    before = [{k: v.clone() for k, v in d.items()} for _, d in s.layers()]
    s.pack()
    for (is_attn, d), ref in zip(s.layers(), before):
        for k, v in ref.items():
            assert torch.equal(d[k], v), k
            base = s.out_dev if k == 'out' else s.in_dev
            assert d[k].untyped_storage().data_ptr() == base.untyped_storage().data_ptr(), k
            assert (d[k].data_ptr() - base.data_ptr()) % 256 == 0, k
    assert s.in_dev.numel() * 4 == sum(v.numel() * 4 for _, d in s.layers()
                                       for k, v in d.items() if k != 'out')


def test_groups_cover_their_four_layers():
    s = _step()
    s.pack()
    layers = list(s.layers())
    assert len(s.in_groups) == len(s.out_groups) == bench.LAYERS // 4
    assert s.in_groups[0][0] == 0 and s.in_groups[-1][1] == s.in_dev.numel()
    for (lo, hi), (nlo, _) in zip(s.in_groups, s.in_groups[1:]):
        assert hi == nlo
    for g, ((lo, hi), (olo, ohi)) in enumerate(zip(s.in_groups, s.out_groups)):
        for is_attn, d in layers[4 * g:4 * g + 4]:
            for k in s.IN_KEYS[is_attn]:
                off = (d[k].data_ptr() - s.in_dev.data_ptr()) // 4
                assert lo <= off and off + d[k].numel() <= hi
            off = (d['out'].data_ptr() - s.out_dev.data_ptr()) // 4
            assert olo <= off and off + d['out'].numel() <= ohi
