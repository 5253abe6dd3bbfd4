"""Optimizer-like wrapper of the native training runtime (odie/native_backend.py).

The public surface the training loop uses (odie/native_backend.py): param_groups, state,
prepare_epoch, train_batch, release_graph, recaptures, build_manifest, state_summary,
native_state_digest, close.  A step is one C-ABI call (odie_step); prepare_epoch captures it,
with the batch's loss, in a CUDA graph that every full batch replays.  The batch is the
configured batch size (the reference fixes 65536), and the reference's compile-time
specialisation (odie/build.py:26-30) is passed as JSON keys.
"""
import contextlib
import json

import torch

from . import _lib


class PlaneState:
    """Per-plane view of the native optimizer state (odie/native_backend.py:7-20)."""

    def __init__(self, backend, planes):
        self.backend = backend
        self.ranges = {}
        offset = 0
        for plane in planes:
            self.ranges[plane] = (offset, offset + plane.numel())
            offset += plane.numel()

    def get(self, plane, default=None):
        if plane not in self.ranges:
            return default
        value = self.backend.state_summary(*self.ranges[plane])
        return {} if value['pristine'] else {'native_adam_state': True}


def target_bytes(target):
    data = getattr(target, 'data', target)
    return data


class NativeOptimizer:
    def __init__(self, model, target, shape, config, planes, half=True, batch=None, head_grad=None, router_grad=None,
                 pipeline=False):
        """pipeline: the runtime's pipeline mode (routed experts on one GPU): a step returns while its backward
        branches still run on the runtime's own streams, and the next step's forward overlaps them; join() (or any
        other call here, each of which joins first) makes the runtime's stream wait for them.  No CUDA graph is
        captured in this mode."""
        self.lib = _lib.library()
        self.pipeline = bool(pipeline)
        self.model, self.target, self.config = model, target, config
        self.half = half
        self.graph = self.key = None
        self.recaptures = 0
        self.batch = int(batch or config.get('batch_size', 65536))
        self.build_manifest = {'library': str(_lib.LIBRARY), 'arch': 'sm_100a',
                               'levels': model.n_levels, 'router': model.gate is not None}
        # the reference trains on a dedicated stream (odie/train.py:73-75); CUDA graphs need a non-default one
        current = torch.cuda.current_stream()
        self.stream = torch.cuda.Stream() if current == torch.cuda.default_stream() else current
        experts = config['representation'] == 'routed_experts'
        grid_params = planes + [model.router_grid] if experts else planes
        self.param_groups = [dict(name='grid', params=grid_params, lr=config['grid_lr'])]
        if model.gate is not None:
            self.param_groups.append(dict(name='gate', params=list(model.gate.parameters()), lr=config['gate_lr']))
        self.param_groups.append(dict(name='decoder', params=list(model.decoder.parameters()), lr=config['decoder_lr']))
        data = target_bytes(target)
        settings = dict(stream=self.stream.cuda_stream, total=model.grid.numel(), width=shape[1], height=shape[0],
                        mode=20 if half else 16, warp_limit=128, rgb=data.data_ptr(), grid=model.grid.data_ptr(),
                        decoder=model.decoder.params.data_ptr(), levels=model.n_levels,
                        router=int(model.gate is not None), gate_k=int(model.gate_coarse_levels_K),
                        softplus=int(config.get('router_output_activation', 'sigmoid') == 'softplus'),
                        rgb8=int(data.dtype == torch.uint8), batch=self.batch, **self.current_settings())
        if model.gate is not None:
            settings['gate'] = model.gate.params.data_ptr()
        if head_grad is not None:
            settings['head_grad'] = head_grad.data_ptr()
        if config['representation'] in ('hash_grid', 'routed_experts'):
            settings['hash_encoding'] = config['hash_encoding']
        if experts:
            settings.update(experts=model.experts_held, router_encoding=config['router_encoding'], router=0,
                            router_grid=model.router_grid.data_ptr(), bands=model.bands, first_band=model.first_band,
                            experts_per_band=model.per_band)
            if model.bands > 1:
                settings.update(full_height=model.image_rows, row_offset=int(config.get('row_offset', 0)))
            if router_grad is not None:
                settings['router_grad'] = router_grad.data_ptr()
        if self.pipeline:
            settings['pipeline'] = 1
        self.handle = self.lib.odie_create(json.dumps(settings).encode())
        if not self.handle:
            raise RuntimeError(_lib.error())
        self.pointers = json.loads(self.lib.odie_pointers(self.handle))
        self.fixed = torch.zeros(self.batch, device='cuda', dtype=torch.int64)  # the captured step's ids
        self.squares = torch.empty(self.batch, device='cuda', dtype=torch.float32)
        self.graph_loss = None
        self._launched = False
        self.state = PlaneState(self, planes)
        from .gpu_residual import attach_runtime
        attach_runtime(model, self)  # the stage boundary decodes this model through the runtime

    def current_settings(self):
        rates = {g['name'] + '_lr': float(g['lr']) for g in self.param_groups}
        if self.config['representation'] in ('hash_grid', 'routed_experts'):
            allocation = getattr(self.model, 'allocation_settings', lambda: None)()
            extra = {'allocation': allocation} if allocation else {}
            return dict(active=self.model.active_prefix, **rates, **extra)
        return dict(active=self.model.active_prefix,
                    **{k: getattr(self.model, k).data_ptr() for k in ('descriptors', 'node_bitmap', 'node_prefix', 'bitmap')},
                    **rates)

    def check(self, code):
        if code:
            raise RuntimeError(_lib.error())

    @contextlib.contextmanager
    def on_stream(self):
        """Run on the runtime's stream, ordered after and before the caller's current stream."""
        caller = torch.cuda.current_stream()
        if caller == self.stream:
            yield
            return
        self.stream.wait_stream(caller)
        with torch.cuda.stream(self.stream):
            yield
        caller.wait_stream(self.stream)

    def step_raw(self, ids, update=True):
        with self.on_stream():
            self.check(self.lib.odie_step(self.handle, ids.data_ptr(), ids.numel(), int(update)))

    def step_stratified(self, seed, step, n, update=True):
        """One step on the stratified batch (seed, step) drawn on the device (odie_step_stratified): the
        reference's stratified_batches (odie/data.py:63-80) fused into the step's input kernel."""
        with self.on_stream():
            self.check(self.lib.odie_step_stratified(self.handle, int(seed), int(step), int(n), int(update)))

    def join(self):
        """The runtime's stream (and the caller's) waits for the branches a pipelined step left running."""
        with self.on_stream():
            self.check(self.lib.odie_join(self.handle))

    def copied(self, name, shape, dtype):
        with self.on_stream():
            self.check(self.lib.odie_join(self.handle))
            result = torch.empty(shape, device='cuda', dtype=dtype)
            self.check(self.lib.odie_copy(result.data_ptr(), self.pointers[name],
                                          result.numel() * result.element_size(), self.stream.cuda_stream))
        return result

    def release_graph(self):
        """Drop the captured step (after a synchronize, so no replay is still running)."""
        torch.cuda.synchronize()
        self.graph = self.key = None
        self.lib.odie_release_contexts(self.handle)

    def _capture(self):
        """Capture one full-batch step plus the loss of its squared errors as a CUDA graph on the runtime's stream.
        The runtime allocates nothing after creation, so the capture needs no preparation beyond having run each
        kernel once (CUDA loads a library's kernels lazily, on their first launch): the first capture of a runtime
        is preceded by one step that updates nothing."""
        if not self._launched:
            with self.on_stream():
                self.check(self.lib.odie_step(self.handle, self.fixed.data_ptr(), self.batch, 0))
            self._launched = True
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            self.check(self.lib.odie_step(self.handle, self.fixed.data_ptr(), self.batch, 1))
            self.check(self.lib.odie_copy(self.squares.data_ptr(), self.pointers['squares'], self.batch * 4,
                                          self.stream.cuda_stream))
            loss = self.squares.sum(dtype=torch.float64) / self.batch
        return graph, loss

    def prepare_epoch(self):
        """Apply the model's current settings (active prefix, layout, allocation, learning rates) and, when they
        changed, capture the step for them."""
        settings = self.current_settings()
        key = json.dumps(settings, sort_keys=True)
        if key == self.key:
            return
        self.release_graph()
        self.check(self.lib.odie_configure(self.handle, json.dumps(settings).encode()))
        if not self.pipeline:  # a pipelined step leaves branches running past its end: nothing to capture
            self.graph, self.graph_loss = self._capture()
        self.lib.odie_pin_contexts(self.handle)
        self.key = key
        self.recaptures += 1

    def train_batch(self, ids):
        """One step on pixel ids; returns the batch's mean squared error (a CUDA fp64 scalar)."""
        n = ids.numel()
        with self.on_stream():
            if self.graph is not None and n == self.batch:
                self.fixed.copy_(ids)
                self.graph.replay()
                return self.graph_loss
            self.check(self.lib.odie_step(self.handle, ids.data_ptr(), n, 1))
            self.check(self.lib.odie_copy(self.squares.data_ptr(), self.pointers['squares'], n * 4,
                                          self.stream.cuda_stream))
            return self.squares[:n].sum(dtype=torch.float64) / n

    def state_summary(self, begin=-1, end=-1):
        """The runtime's optimizer-state summary: {'pristine'} for a grid range, or the state digest (begin < 0)."""
        reply = self.lib.odie_state(self.handle, begin, end)
        if reply is None:
            raise RuntimeError(_lib.error())
        return json.loads(reply)

    def native_state_digest(self):
        return json.dumps(self.state_summary(), sort_keys=True)

    def close(self):
        if not self.handle:
            return
        self.release_graph()
        self.lib.odie_destroy(self.handle)
        self.handle = None

    def decode(self, begin, count, rgb=None, rgb8=None):
        """Decode pixel ids [begin, begin+count) into fp32 and/or u8 RGB device tensors."""
        with self.on_stream():
            self.check(self.lib.odie_decode(self.handle, begin, count, _lib.ptr(rgb), _lib.ptr(rgb8)))

    def call(self, name, *args):
        """Call a runtime entry point (odie_<name>) on this optimizer's stream."""
        with self.on_stream():
            self.check(getattr(self.lib, 'odie_' + name)(self.handle, *args))


def make_native_optimizer(model, target, shape, config):
    planes = [torch.nn.Parameter(model.grid[level['plane_offset']:level['plane_offset'] +
              level['plane_node_capacity'] * level['plane_dim']].detach()) for level in model.layout['levels']]
    return NativeOptimizer(model, target, shape, config, planes), planes
