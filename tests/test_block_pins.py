"""Pin the per-block reference graphs (oracle/ref_harness.cpp ref_trunk_stem /
ref_trunk_block) to the reference's own VisionTrunk::run.

tests/golden/block_pin_<fmt>.npz holds, for blocks 0 (windowed) and 7
(global), the output of the unmodified VisionTrunk::run on a file whose other
31 blocks are exact identities (every weight and bias zero), i.e. the
reference's own block_k(stem(image 0)); see tests/golden/make_golden.py.
The harness runs the stem and block k of the seeded 8-layer file (the same
draws as blocks 0..7 of the 32-layer file) and must reproduce those values
bit for bit.  The per-block GPU parity test (test_gpu_blocks.py) then takes
its block inputs and expected outputs from these graphs.
"""

import numpy as np
import pytest

from conftest import GOLDEN, rel_l2


@pytest.mark.parametrize("fmt", ["f16", "q8_0", "f32"])
def test_block_graphs_equal_reference_trunk(reference, fmt):
    from oracle.pyoracle import reference_path
    from sam3cpp_b200 import synthetic as s
    gold = np.load(GOLDEN / f"block_pin_{fmt}.npz")
    if reference_path().name != "libsam3ref_v4.so":
        pytest.skip("the pins were generated with the AVX-512 build of the reference")
    model = reference.load(s.synthetic_gguf(fmt, layers=8), 0)
    try:
        x0 = model.stem(s.synthetic_image(0))
        stride = int(gold["stride"])
        for k in gold["blocks"]:
            y = model.block(int(k), x0)
            nchw = np.ascontiguousarray(y.T).reshape(-1)      # [1024][5184]: the trunk's NCHW output
            got = nchw[::stride]
            ref = gold[f"block{k}_sample"]
            assert got.shape == ref.shape
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), \
                (fmt, int(k), float(np.abs(got - ref).max()))
            assert abs(float(nchw.astype(np.float64).mean()) - float(gold[f"block{k}_mean"])) < 1e-9
    finally:
        model.close()


def test_q8_0_gemm_operand_rounding_effect(reference):
    """The GPU GEMMs consume Q8_0 weights as fp16(q*d) (converted once at
    load), not the exact q*d of dequantize_row_q8_0 (ggml-quants.c:436-450).
    Measure, with the reference's own F32 arithmetic on block 0 of the seeded
    weights, how far that rounding alone moves one block: the same block with
    exact q*d weights against fp16(q*d) weights, from the same input."""
    import tempfile
    from pathlib import Path
    from sam3cpp_b200 import synthetic as s
    w = s.make_f32_weights(0, layers=1)
    exact, rounded = dict(w), dict(w)
    n_all = n_diff = 0
    for name, arr in w.items():
        if s.tensor_qtype(name, arr, "q8_0") != s.GGML_Q8_0:
            continue
        raw = s.quantize_q8_0_rows(arr).reshape(-1, 34)
        d = raw[:, :2].copy().view(np.float16).astype(np.float64)
        q = raw[:, 2:].view(np.int8).astype(np.float64)
        ex = (q * d).reshape(arr.shape)                     # exact in float32 (<= 19 significant bits)
        h = ex.astype(np.float16).astype(np.float64)
        n_all += ex.size
        n_diff += int((h != ex).sum())
        exact[name] = ex.astype(np.float32)
        rounded[name] = h.astype(np.float32)
    frac = n_diff / n_all
    with tempfile.TemporaryDirectory() as td:
        pe = s.write_gguf(Path(td) / "exact.gguf", exact, "f32")
        pr = s.write_gguf(Path(td) / "rounded.gguf", rounded, "f32")
        me, mr = reference.load(pe, 0), reference.load(pr, 0)
        x = me.stem(s.synthetic_image(0))
        ye, yr = me.block(0, x), mr.block(0, x)
        me.close()
        mr.close()
    out_rel = rel_l2(yr, ye)
    delta_rel = rel_l2(yr - x, ye - x)
    print(f"Q8_0 operand fp16(q*d) != q*d for {frac:.4f} of block-0 weights; "
          f"effect on block 0: output rel_l2 {out_rel:.2e}, contribution rel_l2 {delta_rel:.2e}")
    assert 0.5 < frac < 0.95
    assert out_rel < 5e-4 and delta_rel < 1e-3
