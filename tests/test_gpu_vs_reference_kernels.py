"""The reference's own GPU kernels against this library's, on the same B200 and the same inputs.

The reference's packed-plane query (odie/packed_kernels.cu query_kernel / gradient_kernel), live residual
scoring (odie/residual_cuda.cu accumulate) and exact greedy (odie/native/selection_cuda.cu) are compiled from
their own sources for sm_100a (oracle/build_ref.py) and called through their own entry points beside this
library's C-ABI on identical device buffers.  Each pair must agree (bit for bit where the contract says so) and
this library's side must not be slower; the measured times are printed as one JSON line per kernel
("REFERENCE_KERNEL_TIME ...") for the design notes.  Times are CUDA-event averages after warm-up.
"""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from odie_b200 import _lib
from odie_b200 import layout as host_layout
from odie_b200 import selection as host
from odie_b200 import workloads
from odie_b200.gpu_residual import ResidualAccumulator

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def timed(fn, reps=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / reps


def report(kernel, ours_ms, reference_ms, **extra):
    line = dict(kernel=kernel, ours_ms=ours_ms, reference_ms=reference_ms, speedup=reference_ms / ours_ms, **extra)
    print('REFERENCE_KERNEL_TIME ' + json.dumps(line))
    return line


def reference_library(name):
    path = ROOT / 'oracle' / '_ref' / name
    if not path.exists():
        pytest.skip('reference GPU oracle (oracle/_ref) was not built')
    return path


def div2k_layout(seed=1729):
    """The c2-planes benchmark layout (16 levels, R 8..1020, 3 on-demand levels) and a random fp32 grid."""
    config, supports, dims, caps, _, _ = workloads.c2_planes(seed=seed, batch=1 << 20)
    lay = host_layout.make_layout(config, supports, dims, caps)
    grid = torch.randn(lay['params'], device='cuda') * 0.1
    tensors = [lay[k].cuda() for k in ('descriptors', 'node_bitmap', 'node_prefix', 'bitmap')]
    return lay, grid, tensors


def test_packed_query_forward_and_backward_vs_reference(cuda):
    import importlib.util
    path = reference_library('query/odie_ref_query.so')
    spec = importlib.util.spec_from_file_location('odie_ref_query', path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    lay, grid, (desc, nb, pf, bm) = div2k_layout()
    n, width = 1 << 20, lay['input_width']
    coords = torch.rand((n, 2), device='cuda', generator=torch.Generator('cuda').manual_seed(2))
    lib, stream = _lib.library(), torch.cuda.current_stream().cuda_stream
    features = torch.empty((n, width), dtype=torch.float16, device='cuda')
    visible = torch.empty((n, desc.shape[0]), dtype=torch.bool, device='cuda')

    def ours_forward():
        _lib.check(lib.odie_query_forward(coords.data_ptr(), n, grid.data_ptr(), desc.data_ptr(), desc.shape[0],
                                          nb.data_ptr(), pf.data_ptr(), bm.data_ptr(), width, features.data_ptr(),
                                          visible.data_ptr(), stream))
    ours_forward()
    ref_features, ref_visible = ref.forward(coords, grid, desc, nb, pf, bm, width)
    torch.cuda.synchronize()
    assert torch.equal(features.view(torch.int16), ref_features.view(torch.int16))
    assert torch.equal(visible, ref_visible)
    forward = report('packed query forward (2^20 coords, c2-planes layout)', timed(ours_forward),
                     timed(lambda: ref.forward(coords, grid, desc, nb, pf, bm, width)))
    upstream = (torch.randn((n, width), device='cuda') * 0.01).half()
    gradient = torch.empty(grid.numel(), device='cuda')

    def ours_backward():
        _lib.check(lib.odie_query_backward(coords.data_ptr(), n, upstream.data_ptr(), width, desc.data_ptr(),
                                           desc.shape[0], nb.data_ptr(), pf.data_ptr(), bm.data_ptr(),
                                           gradient.data_ptr(), grid.numel(), stream))
    backward = report('packed query backward (2^20 coords, c2-planes layout)', timed(ours_backward),
                      timed(lambda: ref.backward(coords, upstream, desc, nb, pf, bm, grid.numel())))
    ref_gradient = ref.backward(coords, upstream, desc, nb, pf, bm, grid.numel())
    ours_backward()
    torch.cuda.synchronize()
    scale = ref_gradient.abs().max().item()
    assert (gradient - ref_gradient).abs().max().item() <= 1e-4 * scale, 'the two scatters disagree beyond fp32 order'
    assert forward['speedup'] >= 1.0 and backward['speedup'] >= 1.0


def test_residual_scoring_vs_reference(cuda):
    path = reference_library('libref_residual.so')
    ref = C.CDLL(str(path))
    ref.score_chunk.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int,
                                C.c_void_p, C.c_void_p, C.c_void_p, C.c_bool, C.c_uint64]
    height, width, r = 4096, 4096, 2048
    g = torch.Generator('cuda').manual_seed(3)
    prediction = torch.rand((height * width, 3), device='cuda', generator=g)
    target = torch.randint(0, 256, (height * width, 3), dtype=torch.uint8, device='cuda', generator=g)
    ours, theirs = ResidualAccumulator((height, width), r), ResidualAccumulator((height, width), r)
    stream = torch.cuda.current_stream().cuda_stream
    args = lambda acc: (prediction.data_ptr(), target.data_ptr(), 0, height * width, width, r, 0, r * r,  # noqa
                        acc.x_edges.data_ptr(), acc.y_edges.data_ptr(), acc.totals.data_ptr(), True, stream)
    assert _lib.library().score_chunk(*args(ours)) == 0 and ref.score_chunk(*args(theirs)) == 0
    torch.cuda.synchronize()
    assert torch.equal(ours.totals, theirs.totals), 'residual totals differ from the reference kernel'
    line = report('live residual scoring (4096 x 4096 pixels into 2048^2 cells)',
                  timed(lambda: _lib.library().score_chunk(*args(ours))), timed(lambda: ref.score_chunk(*args(theirs))))
    assert line['speedup'] >= 0.9


def run_greedy(lib, scores, r, cap, chunk, trace=None):
    n, points = r * r, host.align8(r * r)
    sizes, offsets, tree_size = host.tree_shape(n)
    missing = torch.empty(n, dtype=torch.int32, device='cuda')
    chosen = torch.empty(n, dtype=torch.uint8, device='cuda')
    nodes = torch.empty(points, dtype=torch.uint8, device='cuda')
    tree = torch.empty(tree_size, dtype=torch.int32, device='cuda')
    stats = torch.zeros(4, dtype=torch.int64, device='cuda')
    do, ds = torch.from_numpy(offsets).cuda(), torch.from_numpy(sizes).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    assert lib.selection_init(scores.data_ptr(), n, points, missing.data_ptr(), chosen.data_ptr(), nodes.data_ptr(),
                              tree.data_ptr(), stats.data_ptr(), offsets.ctypes.data, sizes.ctypes.data, len(sizes),
                              stream) == 0
    launches = 0
    for _ in range(n // chunk + 2):  # the host reads the status after every launch, as the reference's caller does
        assert lib.selection_chunk(scores.data_ptr(), n, points, r, cap, True, missing.data_ptr(), chosen.data_ptr(),
                                   nodes.data_ptr(), tree.data_ptr(), do.data_ptr(), ds.data_ptr(), len(sizes), chunk,
                                   stats.data_ptr(), None, stream) == 0
        launches += 1
        if stats[2].item():
            break
    end.record()
    torch.cuda.synchronize()
    assert stats[2].item() == 1 and stats[3].item() == 0
    return chosen.cpu().numpy(), start.elapsed_time(end), launches, int(stats[1].item())


def test_exact_greedy_at_gigapixel_resolution_vs_reference(cuda):
    """R = 2048 (the gigapixel stage-boundary level the reference times at 25.5 s on its RTX 3060) with a smooth
    residual field and a node cap that selects about a quarter of a million cells."""
    path = reference_library('libref_selection.so')
    ref = C.CDLL(str(path))
    p, i = C.c_void_p, C.c_int
    ref.selection_init.argtypes = [p, i, i, p, p, p, p, p, p, p, i, C.c_uint64]
    ref.selection_chunk.argtypes = [p, i, i, i, i, C.c_bool, p, p, p, p, p, p, i, i, p, p, C.c_uint64]
    r, cap = 2048, 1 << 20
    field = workloads.pink_noise(r, r, 11)[..., 0].reshape(-1)
    scores = (field - field.min()).double().square().cuda()
    ours, ours_ms, ours_launches, iterations = run_greedy(_lib.library(), scores, r, cap, 512)
    theirs, ref_ms, ref_launches, ref_iterations = run_greedy(ref, scores, r, cap, 512)
    assert np.array_equal(ours, theirs) and iterations == ref_iterations, 'the two greedies chose differently'
    line = report('exact greedy B2, R = 2048, cap 2^20 nodes (512 choices per launch, status read per launch)',
                  ours_ms, ref_ms, iterations=iterations, selected=int(ours.sum()))
    assert line['speedup'] >= 1.0
