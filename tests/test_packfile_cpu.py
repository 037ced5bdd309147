"""Weight-pack files on the CPU: a file written by save_packs reads back bit for bit,
the packs it holds equal the oracle's operands of the reference's quantisation, and a
damaged file is refused with a RuntimeError."""
import numpy as np
import pytest
import torch

from oracle import ee_oracle as orc


class _Pack:
    def __init__(self, w, seed):
        q, s = orc.quantize_weights_int8(w)  # int8 [K, N], fp32 [N]
        self.K, self.N = q.shape
        self.w_i8 = torch.from_numpy(np.ascontiguousarray(q.T))
        self.w_e4m3 = torch.from_numpy(np.ascontiguousarray(orc.weight_e4m3(q).T))
        self.w_f16 = torch.from_numpy(np.ascontiguousarray(orc.weight_f16(q, s).T))
        self.scale = torch.from_numpy(s.astype(np.float32))


def _packs():
    rng = np.random.default_rng(3)
    return {f"layers.{i}.{n}": _Pack((rng.standard_normal((N, K)) * 0.02).astype(np.float16), i)
            for i in range(2) for n, (N, K) in (("gate_proj", (256, 128)), ("down_proj", (128, 256)))}


def test_round_trip_is_bit_exact(pkg, tmp_path):
    pf = pkg.packfile
    packs = _packs()
    path = str(tmp_path / "model.eepack")
    pf.save_packs(path, packs)
    back = pf.load_packs(path)
    assert set(back) == set(packs)
    for name, p in packs.items():
        q = back[name]
        assert (q.K, q.N) == (p.K, p.N)
        for f in ("w_i8", "w_e4m3", "w_f16", "scale"):
            assert torch.equal(getattr(q, f).view(torch.uint8), getattr(p, f).view(torch.uint8)), (name, f)
        wp = q.to_weight_pack()
        assert wp.K == p.K and wp.N == p.N and torch.equal(wp.w_i8, p.w_i8)


def test_damaged_files_are_refused(pkg, tmp_path):
    pf = pkg.packfile
    path = str(tmp_path / "m.eepack")
    pf.save_packs(path, _packs())
    raw = open(path, "rb").read()
    bad = str(tmp_path / "bad.eepack")
    open(bad, "wb").write(b"NOTAPACK" + raw[8:])
    with pytest.raises(RuntimeError, match="bad magic"):
        pf.load_packs(bad)
    open(bad, "wb").write(raw[: len(raw) - 4096])
    with pytest.raises(RuntimeError, match="malformed or truncated"):
        pf.load_packs(bad)


def test_linear_from_pack_views_the_pack(pkg):
    p = _Pack((np.random.default_rng(1).standard_normal((64, 32)) * 0.02).astype(np.float16), 0)
    wp = pkg.WeightPack.from_arrays(p.w_i8, p.w_e4m3, p.w_f16, p.scale)
    lin = pkg.EntropyDispatchedLinear.from_pack(wp, scale_dtype=torch.float16)
    assert lin.weight_int8.shape == (32, 64) and lin.weight_int8.data_ptr() == wp.w_i8.data_ptr()
    assert lin.weight_scale.dtype == torch.float16
    lin.half()  # the conversion build_dispatched_llama applies keeps the pack in place
    assert lin._pack() is wp
