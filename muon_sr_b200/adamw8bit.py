"""bitsandbytes-style blockwise dynamic 8-bit AdamW with BF16 weight SR on the B200 engine.

Drop-in for ``muon_sr.TritonAdamW8bit`` (muon_sr/triton_adamw_8bit.py:102-241): same
arguments, validation errors, state keys and dtypes (``step, format_version=2, block_size,
optim_bits, state1, state2``, plus ``qmap1/qmap2/absmax1/absmax2`` for 8-bit states), same
seeds, and checkpoint loading that keeps uint8 codes and fp32 scales. The update of every
tensor of a group runs in one multi-tensor launch of the single-pass 8-bit kernel.
"""
import math

import torch
from torch.optim import Optimizer

from . import kernels as K


def create_dynamic_map(signed=True):
    """The 256-entry dynamic (signed) / unsigned-dynamic codebook
    (muon_sr/triton_adamw_8bit.py:14-25: per decade i = 0..6, the midpoints of
    linspace(0.1, 1, 2^i + 1) -- 2^(i+1) + 1 for unsigned -- scaled by 10^(i-6), both signs
    for the signed map, plus 0 and 1, sorted)."""
    data = []
    for i in range(7):
        boundaries = torch.linspace(0.1, 1, 2 ** (i if signed else i + 1) + 1, dtype=torch.float32)
        means = (boundaries[:-1] + boundaries[1:]) / 2
        data.extend((10 ** (-6 + i) * means).tolist())
        if signed:
            data.extend((-10 ** (-6 + i) * means).tolist())
    return torch.tensor(sorted(data + [0., 1.]), dtype=torch.float32)


def _cdiv(a, b):
    return (a + b - 1) // b


class TritonAdamW8bit(Optimizer):
    """Dynamic-codebook 8-bit moments, BF16-SR fallback, BF16 weight SR.

    Default blocks contain 256 elements. Tensors below min_8bit_size=4096 use BF16 moments
    with SR. Set group optim_bits=16 to exclude embeddings/other tensors; for_model() creates
    these groups automatically. CUDA, dense contiguous tensors only.
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0., block_size=256,
                 min_8bit_size=4096, optim_bits=8, shard=None):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, block_size=block_size,
                                      min_8bit_size=min_8bit_size, optim_bits=optim_bits))
        self._maps = {}
        self._qtables = {}
        self._shard = shard
        for group in self.param_groups:
            self._validate_group(group)

    @classmethod
    def for_model(cls, model, min_8bit_size=4096, **kwargs):
        """Embeddings (including tied heads) and tensors below min_8bit_size get 16-bit
        states (muon_sr/triton_adamw_8bit.py:119-136)."""
        if 'optim_bits' in kwargs:
            raise ValueError('for_model selects optim_bits per group')
        embeddings = {id(p) for mod in model.modules() if isinstance(mod, torch.nn.Embedding)
                      for p in mod.parameters()}
        groups = {8: [], 16: []}
        for p in model.parameters():
            if p.requires_grad:
                bits = 16 if id(p) in embeddings or p.numel() < min_8bit_size else 8
                groups[bits].append(p)
        return cls([dict(params=params, optim_bits=bits) for bits, params in groups.items() if params],
                   min_8bit_size=min_8bit_size, **kwargs)

    @staticmethod
    def _validate_group(g):
        """muon_sr/triton_adamw_8bit.py:138-150."""
        for key in ('lr', 'eps', 'weight_decay'):
            v = g[key]
            if not isinstance(v, (int, float)) or not math.isfinite(v) or v < 0:
                raise ValueError(f'{key} must be a finite nonnegative scalar')
        if g['eps'] == 0 or len(g['betas']) != 2 or any(not 0 <= b < 1 for b in g['betas']):
            raise ValueError('eps must be positive and betas must be in [0,1)')
        block = g['block_size']
        if not isinstance(block, int) or block < 32 or block > 4096 or block & (block - 1):
            raise ValueError('block_size must be a power of two between 32 and 4096')
        if g['optim_bits'] not in (8, 16) or not isinstance(g['min_8bit_size'], int) or g['min_8bit_size'] < 0:
            raise ValueError('optim_bits must be 8/16; min_8bit_size must be nonnegative')

    def _init_state(self, p, group):
        """muon_sr/triton_adamw_8bit.py:152-165."""
        bits = 16 if p.numel() < group['min_8bit_size'] else group['optim_bits']
        state = dict(step=0, format_version=2, block_size=group['block_size'], optim_bits=bits)
        dtype = torch.uint8 if bits == 8 else torch.bfloat16
        state.update(state1=torch.zeros_like(p, dtype=dtype), state2=torch.zeros_like(p, dtype=dtype))
        if bits == 8:
            if p.device not in self._maps:
                self._maps[p.device] = (create_dynamic_map(True).to(p.device), create_dynamic_map(False).to(p.device))
            state['qmap1'], state['qmap2'] = self._maps[p.device]
            blocks = _cdiv(p.numel(), group['block_size'])
            state['absmax1'] = torch.zeros(blocks, device=p.device, dtype=torch.float32)
            state['absmax2'] = torch.zeros_like(state['absmax1'])
            state['state1'].fill_(127)  # signed codebook's exact zero
        return state

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self._shard:
            self._shard.bind(self)
        index = 0
        for gi, group in enumerate(self.param_groups):
            self._validate_group(group)
            b1, b2 = group['betas']
            by_maps = {}
            for pi, p in enumerate(group['params']):
                param_index = index
                index += 1
                if p.grad is None:
                    continue
                if p.dtype != torch.bfloat16 or not p.is_cuda:
                    raise ValueError('TritonAdamW8bit requires CUDA BF16 parameters')
                g = p.grad
                if g.is_sparse or not p.is_contiguous() or not g.is_contiguous():
                    raise ValueError('Parameters/gradients must be contiguous and dense')
                if not p.numel():
                    continue
                state = self.state[p]
                if not state:
                    state.update(self._init_state(p, group))
                expected_bits = 16 if p.numel() < group['min_8bit_size'] else group['optim_bits']
                if state['block_size'] != group['block_size'] or state['optim_bits'] != expected_bits:
                    raise ValueError('Cannot change quantization configuration after state initialization')
                state['step'] += 1
                n = state['step']
                if self._shard and not self._shard.owns(gi, pi):
                    continue
                seed = (n * 2654435761 ^ param_index * 1234567891) & 0xFFFFFFFF
                quant = state['optim_bits'] == 8
                maps = (state['qmap1'], state['qmap2']) if quant else (None, None)
                key = (maps[0].data_ptr(), maps[1].data_ptr()) if quant else None
                by_maps.setdefault(key, (maps, []))[1].append(
                    (p, g, state['state1'], state['state2'], state.get('absmax1'), state.get('absmax2'), n, seed,
                     quant))
            for maps, items in by_maps.values():
                tables = None
                if maps[0] is not None:
                    tkey = (maps[0].data_ptr(), maps[1].data_ptr())
                    if tkey not in self._qtables:  # built once per codebook pair (host copy of 2 KB)
                        self._qtables[tkey] = K.quant_tables(maps[0], maps[1])
                    tables = self._qtables[tkey]
                K.adamw8bit(items, maps[0], maps[1], group['lr'], b1, b2, group['eps'], group['weight_decay'],
                            group['block_size'], qtables=tables)
        if self._shard:
            self._shard.sync_params(self)
        return loss

    def load_state_dict(self, state_dict):
        """Keeps uint8 codes and fp32 scales and validates the checkpoint
        (muon_sr/triton_adamw_8bit.py:207-241)."""
        groups = state_dict['param_groups']
        if len(groups) != len(self.param_groups) or any(
                len(a['params']) != len(b['params']) for a, b in zip(groups, self.param_groups)):
            raise ValueError('Checkpoint parameter groups do not match optimizer')
        mapping = dict(zip([i for g in groups for i in g['params']],
                           [p for g in self.param_groups for p in g['params']]))
        restored = {}
        keys = {'state1', 'state2', 'qmap1', 'qmap2', 'absmax1', 'absmax2'}
        for group in groups:
            self._validate_group(group)
            for ident in group['params']:
                state = state_dict['state'].get(ident, {})
                if not state:
                    continue
                p = mapping[ident]
                bits = 16 if p.numel() < group['min_8bit_size'] else group['optim_bits']
                if state.get('format_version') != 2 or state.get('block_size') != group['block_size'] or \
                        state.get('optim_bits') != bits:
                    raise ValueError('Incompatible state format/quantization configuration')
                specs = {key: (p.shape, torch.uint8 if bits == 8 else torch.bfloat16) for key in ('state1', 'state2')}
                if bits == 8:
                    specs.update({key: ((256,), torch.float32) for key in ('qmap1', 'qmap2')})
                    specs.update({key: ((_cdiv(p.numel(), group['block_size']),), torch.float32)
                                  for key in ('absmax1', 'absmax2')})
                restored[ident] = {}
                for key, (shape, dtype) in specs.items():
                    value = state[key]
                    if value.dtype != dtype or tuple(value.shape) != tuple(shape):
                        raise ValueError(f'Invalid checkpoint state: {key}')
                    restored[ident][key] = value.to(device=p.device, dtype=dtype).clone()
        stripped = dict(state_dict, state={i: {k: v for k, v in state.items() if k not in keys}
                                           for i, state in state_dict['state'].items()})
        super().load_state_dict(stripped)
        for ident, values in restored.items():
            self.state[mapping[ident]].update(values)
