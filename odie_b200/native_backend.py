"""Optimizer-like wrapper of the native training runtime (odie/native_backend.py).

Same public surface as the reference's NativeOptimizer: param_groups, state,
prepare_epoch, train_batch, release_graph, recaptures, build_manifest,
state_summary, native_state_digest, close.  The step is one C-ABI call
(odie_step) captured in a CUDA graph and replayed for every full batch.
Differences from the reference: the batch is the configured batch size (not
fixed at 65536) and the compile-time specialisation of the reference build
(odie/build.py:26-30) is passed as JSON keys.
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
    def __init__(self, model, target, shape, config, planes, half=True, batch=None, head_grad=None):
        self.lib = _lib.library()
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
            settings.update(experts=model.experts, router_encoding=config['router_encoding'], router=0,
                            router_grid=model.router_grid.data_ptr())
        self.handle = self.lib.odie_create(json.dumps(settings).encode())
        if not self.handle:
            raise RuntimeError(_lib.error())
        self.pointers = json.loads(self.lib.odie_pointers(self.handle))
        self.fixed = torch.zeros(self.batch, device='cuda', dtype=torch.int64)
        self.squares = torch.empty(self.batch, device='cuda', dtype=torch.float32)
        self.state = PlaneState(self, planes)

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

    def copied(self, name, shape, dtype):
        with self.on_stream():
            result = torch.empty(shape, device='cuda', dtype=dtype)
            self.check(self.lib.odie_copy(result.data_ptr(), self.pointers[name],
                                          result.numel() * result.element_size(), self.stream.cuda_stream))
        return result

    def release_graph(self):
        torch.cuda.synchronize()
        self.graph = self.key = None
        self.lib.odie_release_contexts(self.handle)

    def prepare_epoch(self):
        settings = self.current_settings()
        key = tuple(settings.items())
        if key == self.key:
            return
        self.release_graph()
        self.check(self.lib.odie_configure(self.handle, json.dumps(settings).encode()))
        for _ in range(3):
            self.step_raw(self.fixed, update=False)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            self.check(self.lib.odie_step(self.handle, self.fixed.data_ptr(), self.fixed.numel(), 1))
            self.check(self.lib.odie_copy(self.squares.data_ptr(), self.pointers['squares'], self.batch * 4,
                                          self.stream.cuda_stream))
            self.graph_loss = self.squares.double().mean()
        self.lib.odie_pin_contexts(self.handle)
        self.graph, self.key = graph, key
        self.recaptures += 1

    def train_batch(self, ids):
        with self.on_stream():
            if ids.numel() == self.batch and self.graph is not None:
                self.fixed.copy_(ids)
                self.graph.replay()
                return self.graph_loss
            self.check(self.lib.odie_step(self.handle, ids.data_ptr(), ids.numel(), 1))
            self.check(self.lib.odie_copy(self.squares.data_ptr(), self.pointers['squares'], ids.numel() * 4,
                                          self.stream.cuda_stream))
            return self.squares[:ids.numel()].double().mean()

    def state_summary(self, begin=-1, end=-1):
        data = self.lib.odie_state(self.handle, begin, end)
        if data is None:
            raise RuntimeError(_lib.error())
        return json.loads(data)

    def native_state_digest(self):
        return json.dumps(self.state_summary(), sort_keys=True)

    def close(self):
        if self.handle:
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
