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
from . import staging


def create_dynamic_map(signed=True):
    """The 256-entry dynamic codebook of ``muon_sr.triton_adamw_8bit.create_dynamic_map``
    (triton_adamw_8bit.py:14-25), bit for bit.

    Decade k = 0..6 covers [0.1, 1) x 10^(k-6) with the midpoints of an fp32 ``linspace``
    grid of 2^k intervals (2^(k+1) for the unsigned map, which has no negative half); the
    signed map mirrors every value; 0 and 1 are added and the table is sorted."""
    half = []
    for decade in range(7):
        intervals = 1 << (decade if signed else decade + 1)
        edges = torch.linspace(0.1, 1, intervals + 1, dtype=torch.float32)
        mids = (edges[:-1] + edges[1:]) / 2
        half.append(10 ** (decade - 6) * mids)
    pos = torch.cat(half)
    table = torch.cat([pos, -pos]) if signed else pos
    table = torch.cat([table, torch.tensor([0.0, 1.0])])
    return table.sort().values.to(torch.float32)


def _blocks(numel, block):
    return -(-numel // block)


def _bits_for(p, group):
    """Moment width of a parameter: tensors below min_8bit_size always keep bf16 moments."""
    return 16 if p.numel() < group['min_8bit_size'] else group['optim_bits']


def _state_spec(p, group):
    """(shape, dtype) of every tensor the optimizer keeps for ``p`` -- one definition for
    state creation and checkpoint validation."""
    if _bits_for(p, group) == 16:
        return {'state1': (tuple(p.shape), torch.bfloat16), 'state2': (tuple(p.shape), torch.bfloat16)}
    nblk = (_blocks(p.numel(), group['block_size']),)
    return {'state1': (tuple(p.shape), torch.uint8), 'state2': (tuple(p.shape), torch.uint8),
            'qmap1': ((256,), torch.float32), 'qmap2': ((256,), torch.float32),
            'absmax1': (nblk, torch.float32), 'absmax2': (nblk, torch.float32)}


_TENSOR_KEYS = ('state1', 'state2', 'qmap1', 'qmap2', 'absmax1', 'absmax2')


def _check_group(g):
    """The reference's group rules (triton_adamw_8bit.py:138-150), raising ValueError."""
    for key in ('lr', 'eps', 'weight_decay'):
        v = g[key]
        if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v) or v < 0:
            raise ValueError(f'{key} must be a finite number >= 0, got {v!r}')
    if g['eps'] == 0:
        raise ValueError('eps must be positive')
    betas = g['betas']
    if len(betas) != 2 or not all(0 <= b < 1 for b in betas):
        raise ValueError(f'betas must be two values in [0, 1), got {betas!r}')
    block = g['block_size']
    if not isinstance(block, int) or not 32 <= block <= 4096 or block & (block - 1):
        raise ValueError(f'block_size must be a power of two in [32, 4096], got {block!r}')
    if g['optim_bits'] not in (8, 16):
        raise ValueError(f"optim_bits must be 8 or 16, got {g['optim_bits']!r}")
    if not isinstance(g['min_8bit_size'], int) or g['min_8bit_size'] < 0:
        raise ValueError(f"min_8bit_size must be an int >= 0, got {g['min_8bit_size']!r}")


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
            _check_group(group)

    @classmethod
    def for_model(cls, model, min_8bit_size=4096, **kwargs):
        """Two groups: 16-bit moments for embedding weights (a tied output head is the same
        tensor) and tensors below min_8bit_size, 8-bit for the rest
        (triton_adamw_8bit.py:119-136)."""
        if 'optim_bits' in kwargs:
            raise ValueError('for_model chooses optim_bits itself; pass it per group to the constructor instead')
        embedding_ids = set()
        for module in model.modules():
            if isinstance(module, torch.nn.Embedding):
                embedding_ids.update(id(t) for t in module.parameters())
        wide, narrow = [], []
        for t in model.parameters():
            if not t.requires_grad:
                continue
            (wide if id(t) in embedding_ids or t.numel() < min_8bit_size else narrow).append(t)
        groups = [dict(params=ts, optim_bits=bits) for bits, ts in ((8, narrow), (16, wide)) if ts]
        return cls(groups, min_8bit_size=min_8bit_size, **kwargs)

    def _codebooks(self, device):
        if device not in self._maps:
            self._maps[device] = (create_dynamic_map(True).to(device), create_dynamic_map(False).to(device))
        return self._maps[device]

    def _init_state(self, p, group):
        """Fresh state (triton_adamw_8bit.py:152-165): zero moments -- code 127 is the signed
        codebook's exact zero, code 0 the unsigned one's -- and zero block scales."""
        spec = _state_spec(p, group)
        state = dict(step=0, format_version=2, block_size=group['block_size'], optim_bits=_bits_for(p, group))
        for key in ('state1', 'state2', 'absmax1', 'absmax2'):
            if key in spec:
                shape, dtype = spec[key]
                state[key] = torch.zeros(shape, dtype=dtype, device=p.device)
        if 'qmap1' in spec:
            state['qmap1'], state['qmap2'] = self._codebooks(p.device)
            state['state1'].fill_(127)
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
            _check_group(group)
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
                if state['block_size'] != group['block_size'] or state['optim_bits'] != _bits_for(p, group):
                    raise ValueError('block_size / optim_bits of a group changed after its state was created')
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
                for part in staging.batches(items, lambda e: e[0].numel()):
                    staging.need([e[0] for e in part])
                    K.adamw8bit(part, maps[0], maps[1], group['lr'], b1, b2, group['eps'], group['weight_decay'],
                                group['block_size'], qtables=tables)
                    staging.done([e[0] for e in part])
        if self._shard:
            self._shard.sync_params(self)
        return loss

    def load_state_dict(self, state_dict):
        """Checkpoint loading that keeps uint8 codes and fp32 scales (torch's default would cast
        every state tensor to the parameter's dtype) and rejects checkpoints whose layout does
        not match this optimizer's groups (triton_adamw_8bit.py:207-241)."""
        saved_groups = state_dict['param_groups']
        if [len(g['params']) for g in saved_groups] != [len(g['params']) for g in self.param_groups]:
            raise ValueError('checkpoint param groups do not match this optimizer')
        param_of = {}
        for saved, live in zip(saved_groups, self.param_groups):
            param_of.update(zip(saved['params'], live['params']))
        kept = {}
        for saved in saved_groups:
            _check_group(saved)
            for ident in saved['params']:
                st = state_dict['state'].get(ident)
                if not st:
                    continue
                p = param_of[ident]
                layout = (st.get('format_version'), st.get('block_size'), st.get('optim_bits'))
                if layout != (2, saved['block_size'], _bits_for(p, saved)):
                    raise ValueError(f'checkpoint state of parameter {ident} has an incompatible layout {layout}')
                kept[ident] = {}
                for key, (shape, dtype) in _state_spec(p, saved).items():
                    t = st[key]
                    if t.dtype != dtype or tuple(t.shape) != shape:
                        raise ValueError(f'checkpoint tensor {key} of parameter {ident} has dtype {t.dtype} and '
                                         f'shape {tuple(t.shape)}, expected {dtype} {shape}')
                    kept[ident][key] = t.to(device=p.device).clone()
        rest = {i: {k: v for k, v in st.items() if k not in _TENSOR_KEYS} for i, st in state_dict['state'].items()}
        super().load_state_dict(dict(state_dict, state=rest))
        for ident, tensors in kept.items():
            self.state[param_of[ident]].update(tensors)
