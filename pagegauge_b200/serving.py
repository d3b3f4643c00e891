"""Served cache layout: PageGauge kernels on a paged serving pool.

Mirrors the reference's serving package
(experiments/mlsys2027/serving_v1/pagegauge_vllm/) with the same names,
arguments, results and error messages, and adds the device side that the
reference leaves to a future engine: the fused append and the decode run
directly on the pool, addressed by the decode metadata's integer columns.

* ``Policy``, ``partition``, ``exact_slot`` -- page-aligned prefix (S) /
  static prompt suffix (A) / tail ring (T) semantics (partition.py:1-52).
* ``Layout`` -- capacity accounting of the persistent code pool plus every
  admitted request's exact and centre sidecars, and the pages a cache
  budget admits (cache_layout.py:6-38).
* ``dense_pool_views``, ``from_engine_layer``, ``zero_physical_pages`` --
  one raw uint8 allocation per layer split into whole-pool K codes, V codes,
  K scales and V scales planes, zero-copy (cache_views.py:9-62).  The
  planes are exactly the dense [pages, 16, Hkv, 128] codes and [pages, Hkv]
  scales the decode kernels read, so the pool plugs in without a repack.
* ``allocate_sidecars`` -- exact pages [L, R*storage, 16, Hkv, 128] and
  centres [L, R, Hkv, 128] (sidecars.py:10-35).
* ``RequestSlots`` / ``Lease`` / ``State`` -- explicit request lifetimes,
  lease generations, page ownership (request_slots.py:1-93).
* ``prepare_decode`` / ``commit_decode`` / ``DecodeBatch`` -- the decode
  batch metadata and its commit (decode_metadata.py:1-76).
* ``ServedPool`` -- the GPU side: a model's pool and sidecars, prompt
  packing, and the served decode step (per layer: one fused RoPE + centred
  append + page close on the pool slots, then the split-KV PageGauge decode
  over the request's history pages in the pool and exact pages in the
  sidecar).

Pages close to INT8 when their 16th token is appended, so a page that later
ages out of the tail ring already has its codes in the pool; the aged pages
``prepare_decode`` reports need no further device work.
"""

from __future__ import annotations

import heapq
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

PAGE = 16


# ----------------------------------------------------------------- policy
@dataclass(frozen=True)
class Policy:
    """S/A/T page policy: ``prefix_pages`` exact pages at the start,
    ``suffix_pages`` exact pages that ended the prompt, and a tail ring of
    ``tail_pages`` (partition.py:7-18)."""
    prefix_pages: int = 4
    suffix_pages: int = 128
    tail_pages: int = 48

    def __post_init__(self):
        values = (self.prefix_pages, self.suffix_pages, self.tail_pages)
        if (any(type(v) is not int for v in values) or self.prefix_pages < 0
                or self.suffix_pages < 0 or self.tail_pages < 1):
            raise ValueError('Invalid page policy')

    @property
    def storage_pages(self) -> int:
        return self.prefix_pages + self.suffix_pages + self.tail_pages


def partition(prompt_tokens, current_tokens, policy: Policy = Policy()) -> dict:
    """Logical pages of a request with ``current_tokens`` tokens split into
    exact (prefix, suffix, tail) and history (INT8) pages
    (partition.py:21-40).  The partial last prompt page belongs to the tail."""
    if (type(prompt_tokens) is not int or type(current_tokens) is not int
            or not 0 < prompt_tokens <= current_tokens):
        raise ValueError('Invalid prompt/current length')
    initial = prompt_tokens // PAGE
    pages = -(-current_tokens // PAGE)
    if (initial < policy.prefix_pages + policy.suffix_pages
            or pages - policy.tail_pages <= policy.prefix_pages):
        raise ValueError('Prompt cannot support this policy; explicit FP16 fallback required')
    prefix = range(policy.prefix_pages)
    suffix = range(initial - policy.suffix_pages, initial)
    tail = range(pages - policy.tail_pages, pages)
    exact = sorted(set(prefix) | set(suffix) | set(tail))
    exact_set = set(exact)
    history = tuple(p for p in range(pages) if p not in exact_set)
    if not history or history[-1] == pages - 1:
        raise ValueError('No historical page or partial last page incorrectly quantized')
    return {'prefix': tuple(prefix), 'suffix': tuple(suffix), 'tail': tuple(tail),
            'exact': tuple(exact), 'history': history,
            'history_tokens': PAGE * len(history),
            'exact_tokens': current_tokens - PAGE * len(history),
            'tail_tokens': (policy.tail_pages - 1) * PAGE + (current_tokens - 1) % PAGE + 1}


def exact_slot(logical_page, prompt_tokens, lease_slot, policy: Policy = Policy()) -> int:
    """Sidecar page of an exact logical page: prefix pages in order, then the
    suffix pages, then the tail ring slot ``page % tail_pages``
    (partition.py:43-52)."""
    initial = prompt_tokens // PAGE
    if min(logical_page, lease_slot) < 0:
        raise ValueError('Negative page/lease slot')
    if logical_page < policy.prefix_pages:
        local = logical_page
    elif initial - policy.suffix_pages <= logical_page < initial:
        local = policy.prefix_pages + logical_page - (initial - policy.suffix_pages)
    else:
        local = policy.prefix_pages + policy.suffix_pages + logical_page % policy.tail_pages
    return lease_slot * policy.storage_pages + local


# ---------------------------------------------------------------- layout
@dataclass(frozen=True)
class Layout:
    """Served pool geometry and its capacity accounting (cache_layout.py)."""
    layers: int
    physical_pages: int
    maximum_requests: int
    kv_heads: int = 8
    query_heads: int = 32
    head_dim: int = 128
    policy: Policy = Policy()

    def __post_init__(self):
        geometry = (self.layers, self.physical_pages, self.maximum_requests, self.kv_heads,
                    self.query_heads, self.head_dim)
        if (any(type(v) is not int or v < 1 for v in geometry)
                or self.query_heads % self.kv_heads):
            raise ValueError('Invalid cache geometry')

    def accounting(self) -> dict:
        L, N, R = self.layers, self.physical_pages, self.maximum_requests
        H, Q, D = self.kv_heads, self.query_heads, self.head_dim
        codes = L * N * PAGE * H * D
        exact = 2 * L * R * self.policy.storage_pages * PAGE * H * D
        tensors = {'key_codes': codes, 'value_codes': codes,
                   'key_scales': 2 * L * N * H, 'value_scales': 2 * L * N * H,
                   'exact_key': exact, 'exact_value': exact,
                   'key_center': 2 * L * R * H * D, 'value_center': 2 * L * R * H * D,
                   'output_center': 2 * L * R * Q * D}
        pool = sum(tensors[k] for k in ('key_codes', 'value_codes', 'key_scales', 'value_scales'))
        total = sum(tensors.values())
        return {'tensors': tensors, 'page_pool_bytes': pool,
                'reserved_sidecar_bytes': total - pool,
                'total_served_capacity_bytes': total,
                'per_layer_page_bytes': 2 * PAGE * H * D + 4 * H,
                'scope': ('Declared persistent code/metadata pool and all admitted-request '
                          'sidecar slots, including empty reserved slots. Excludes weights, '
                          'workspace, graph pools, input/output buffers and allocator padding; '
                          'those must be separately reserved/measured before admission.')}

    def admissible_pages(self, cache_budget_bytes) -> int:
        """Physical pages a cache-only byte budget holds after every
        reserved sidecar (cache_layout.py:33-38)."""
        acc = self.accounting()
        remaining = cache_budget_bytes - acc['reserved_sidecar_bytes']
        if remaining < 0:
            raise MemoryError('Budget cannot hold reserved exact/center sidecars')
        return remaining // (self.layers * acc['per_layer_page_bytes'])

    @classmethod
    def for_budget(cls, layers: int, maximum_requests: int, cache_budget_bytes: int,
                   **kw) -> "Layout":
        """The largest pool a cache-only budget admits (e.g. a B200's HBM
        minus weights, workspace and graph pools)."""
        probe = cls(layers, 1, maximum_requests, **kw)
        pages = probe.admissible_pages(cache_budget_bytes)
        if pages < 1:
            raise MemoryError('Budget cannot hold reserved exact/center sidecars')
        return cls(layers, int(pages), maximum_requests, **kw)


# ----------------------------------------------------------------- views
def dense_pool_views(raw: torch.Tensor, physical_pages, kv_heads, head_dim=128) -> dict:
    """Split one layer's raw uint8 allocation into the K codes, V codes, K
    scales and V scales planes, without a copy (cache_views.py:9-24)."""
    if any(type(x) is not int or x < 1 for x in (physical_pages, kv_heads, head_dim)):
        raise ValueError('Positive integer pool geometry required')
    codes = physical_pages * PAGE * kv_heads * head_dim
    scales = physical_pages * kv_heads * 2
    if (raw.dtype != torch.uint8 or raw.ndim != 1 or not raw.is_contiguous()
            or raw.numel() != 2 * codes + 2 * scales or raw.data_ptr() % 16):
        raise ValueError('Aligned contiguous uint8 layer allocation of exact size required')
    return {
        'key_codes': raw[:codes].view(torch.int8).view(physical_pages, PAGE, kv_heads, head_dim),
        'value_codes': raw[codes:2 * codes].view(torch.int8).view(physical_pages, PAGE, kv_heads,
                                                                   head_dim),
        'key_scales': raw[2 * codes:2 * codes + scales].view(torch.float16).view(physical_pages,
                                                                                 kv_heads),
        'value_scales': raw[2 * codes + scales:].view(torch.float16).view(physical_pages,
                                                                          kv_heads),
    }


def from_engine_layer(layer: torch.Tensor, physical_pages, kv_heads) -> dict:
    """Reinterpret a compact packed engine layer [pages, Hkv, 1, 2*16*128+4]
    uint8 as pool planes, no copy (cache_views.py:27-39)."""
    expected = (physical_pages, kv_heads, 1, 2 * PAGE * 128 + 4)
    if layer.dtype != torch.uint8 or tuple(layer.shape) != expected or not layer.is_contiguous():
        raise ValueError('Compact packed engine layer required; copying is forbidden')
    return dense_pool_views(layer.view(-1), physical_pages, kv_heads)


def zero_physical_pages(views: dict, page_ids) -> None:
    """Zero the four planes of the given pool pages on the current stream,
    one kernel launch (cache_views.py:42-62)."""
    names = ('key_codes', 'value_codes', 'key_scales', 'value_scales')
    tensors = [views[n] for n in names]
    first = tensors[0]
    pages = tuple(page_ids)
    if (any(t.device != first.device or t.shape[0] != first.shape[0] for t in tensors)
            or any(type(p) is not int or not 0 <= p < first.shape[0] for p in pages)
            or len(set(pages)) != len(pages)):
        raise ValueError('Invalid physical pages or inconsistent pool views')
    if not pages:
        return
    if not first.is_cuda:
        raise ValueError('pool views must be CUDA tensors')
    ids = torch.tensor(pages, dtype=torch.int32).to(first.device, non_blocking=True)
    _lib.call('pg_zero_pool_pages', first.data_ptr(), tensors[1].data_ptr(),
              tensors[2].data_ptr(), tensors[3].data_ptr(), first.shape[0], first.shape[2],
              ids.data_ptr(), len(pages), torch.cuda.current_stream(first.device).cuda_stream)


def allocate_sidecars(layout: Layout, *, device, cache_budget_bytes) -> dict:
    """Exact pages and centres reserved for every admissible request
    (sidecars.py:10-35)."""
    if type(cache_budget_bytes) is not int or cache_budget_bytes < 0:
        raise ValueError('Nonnegative integer cache-only byte budget required')
    acc = layout.accounting()
    if acc['total_served_capacity_bytes'] > cache_budget_bytes:
        raise MemoryError('Code pool plus all reserved sidecars exceed cache budget')
    L, R, H, D = layout.layers, layout.maximum_requests, layout.kv_heads, layout.head_dim
    exact = (L, R * layout.policy.storage_pages, PAGE, H, D)
    shapes = {'exact_key': exact, 'exact_value': exact, 'key_center': (L, R, H, D),
              'value_center': (L, R, H, D), 'output_center': (L, R, layout.query_heads, D)}
    out = {name: torch.zeros(shape, dtype=torch.float16, device=device)
           for name, shape in shapes.items()}
    for name, t in out.items():
        if t.numel() * t.element_size() != acc['tensors'][name]:
            raise RuntimeError('Sidecar allocation differs from declared accounting')
    return out


# ------------------------------------------------------- request lifetimes
@dataclass(frozen=True)
class Lease:
    request_id: str
    slot: int
    generation: int


@dataclass(frozen=True)
class State:
    lease: Lease
    prompt_tokens: int
    current_tokens: int
    physical_pages: tuple


class RequestSlots:
    """Fixed admission capacity of sidecar slots; a request holds a lease
    (slot + generation) and owns its physical pages until released
    (request_slots.py:20-93)."""

    def __init__(self, maximum_requests, policy: Policy = Policy()):
        if type(maximum_requests) is not int or maximum_requests < 1:
            raise ValueError('Positive fixed admission capacity required')
        self.policy = policy
        self.free = list(range(maximum_requests))
        self.generations = [0] * maximum_requests
        self.states: dict[str, State] = {}
        self.page_owner: dict[int, Lease] = {}

    def _pages(self, physical_pages, count) -> tuple:
        pages = tuple(physical_pages)
        if (len(pages) != count or len(set(pages)) != count
                or any(type(p) is not int or p < 0 for p in pages)):
            raise ValueError('Wrong/duplicate physical block table')
        return pages

    def admit(self, request_id, prompt_tokens, physical_pages) -> Lease:
        if not isinstance(request_id, str) or not request_id or request_id in self.states:
            raise ValueError('Invalid or duplicate live request ID')
        partition(prompt_tokens, prompt_tokens, self.policy)
        pages = self._pages(physical_pages, -(-prompt_tokens // PAGE))
        if any(p in self.page_owner for p in pages):
            raise ValueError('Cross-request page sharing is disabled')
        if not self.free:
            raise MemoryError('Declared exact-sidecar admission capacity reached')
        slot = heapq.heappop(self.free)
        self.generations[slot] += 1
        lease = Lease(request_id, slot, self.generations[slot])
        self.states[request_id] = State(lease, prompt_tokens, prompt_tokens, pages)
        for p in pages:
            self.page_owner[p] = lease
        return lease

    def state(self, lease: Lease) -> State:
        st = self.states.get(lease.request_id)
        if st is None or st.lease != lease:
            raise ValueError('Stale request lease/center generation')
        return st

    def batch(self, request_ids) -> tuple:
        ids = tuple(request_ids)
        if len(set(ids)) != len(ids):
            raise ValueError('Duplicate batch row')
        try:
            return tuple(self.states[i].lease for i in ids)
        except KeyError as error:
            raise ValueError('Unknown scheduled request') from error

    def append(self, lease: Lease, position, physical_pages) -> dict:
        st = self.state(lease)
        if position != st.current_tokens:
            raise ValueError('Skipped/replayed token or wrong per-request position')
        length = position + 1
        pages = self._pages(physical_pages, -(-length // PAGE))
        if pages[:len(st.physical_pages)] != st.physical_pages:
            raise ValueError('Preemption/remapping is not supported in phase one')
        extra = pages[len(st.physical_pages):]
        if any(p in self.page_owner for p in extra):
            raise ValueError('New physical page belongs to a live request')
        before = partition(st.prompt_tokens, st.current_tokens, self.policy)
        after = partition(st.prompt_tokens, length, self.policy)
        aged = sorted(set(after['history']) - set(before['history']))
        if any(p >= length // PAGE for p in aged):
            raise ValueError('Attempt to consume an unfinished INT8 page')
        for p in extra:
            self.page_owner[p] = lease
        self.states[lease.request_id] = State(lease, st.prompt_tokens, length, pages)
        return {'lease': lease, 'position': position,
                'closed_page': position // PAGE if length % PAGE == 0 else None,
                'new_history_pages': tuple(aged), 'partition': after}

    def release(self, lease: Lease) -> None:
        st = self.state(lease)
        if any(self.page_owner.get(p) != lease for p in st.physical_pages):
            raise ValueError('Page ownership corrupted')
        for p in st.physical_pages:
            del self.page_owner[p]
        del self.states[lease.request_id]
        heapq.heappush(self.free, lease.slot)


# ------------------------------------------------------- decode metadata
@dataclass(frozen=True)
class DecodeRow:
    lease: Lease
    expected_state: State
    position: int
    physical_pages: tuple
    physical_token_slot: int
    exact_token_slot: int
    new_history_logical_pages: tuple
    new_history_physical_pages: tuple
    new_history_exact_slots: tuple


@dataclass(frozen=True)
class DecodeBatch:
    rows: tuple

    def columns(self) -> dict:
        """Integer columns of the device ABI, in scheduled row order
        (decode_metadata.py:28-35)."""
        return {'request_slots': tuple(r.lease.slot for r in self.rows),
                'generations': tuple(r.lease.generation for r in self.rows),
                'positions': tuple(r.position for r in self.rows),
                'physical_token_slots': tuple(r.physical_token_slot for r in self.rows),
                'exact_token_slots': tuple(r.exact_token_slot for r in self.rows)}


def prepare_decode(manager: RequestSlots, scheduled) -> DecodeBatch:
    """Validate a batch of (lease, next position, full physical block table)
    without mutating the manager (decode_metadata.py:38-62)."""
    rows = []
    ids = set()
    allocated = set(manager.page_owner)
    for lease, position, physical_pages in scheduled:
        st = manager.state(lease)
        if lease.request_id in ids:
            raise ValueError('Duplicate scheduled request')
        ids.add(lease.request_id)
        if type(position) is not int or position != st.current_tokens:
            raise ValueError('Wrong next token position')
        pages = manager._pages(physical_pages, (position + PAGE) // PAGE)
        if pages[:len(st.physical_pages)] != st.physical_pages:
            raise ValueError('Physical remapping is unsupported')
        extra = pages[len(st.physical_pages):]
        if any(p in allocated for p in extra):
            raise ValueError('Physical page alias across batch')
        allocated.update(extra)
        before = partition(st.prompt_tokens, position, manager.policy)
        after = partition(st.prompt_tokens, position + 1, manager.policy)
        aged = tuple(sorted(set(after['history']) - set(before['history'])))
        if any(p >= (position + 1) // PAGE for p in aged):
            raise ValueError('Cannot quantize incomplete page')
        page = position // PAGE
        rows.append(DecodeRow(
            lease, st, position, pages, pages[page] * PAGE + position % PAGE,
            exact_slot(page, st.prompt_tokens, lease.slot, manager.policy) * PAGE
            + position % PAGE,
            aged, tuple(pages[p] for p in aged),
            tuple(exact_slot(p, st.prompt_tokens, lease.slot, manager.policy) for p in aged)))
    return DecodeBatch(tuple(rows))


def commit_decode(manager: RequestSlots, batch: DecodeBatch) -> tuple:
    """Advance the manager after the batch's device work has completed
    (decode_metadata.py:65-76)."""
    for row in batch.rows:
        if manager.state(row.lease) != row.expected_state:
            raise ValueError('Decode batch is stale')
    fresh = prepare_decode(manager, [(r.lease, r.position, r.physical_pages) for r in batch.rows])
    if fresh != batch:
        raise ValueError('Decode metadata was altered')
    return tuple(manager.append(r.lease, r.position, r.physical_pages) for r in batch.rows)


def decode_tables(batch: DecodeBatch, policy: Policy):
    """Host CSR page tables of a decode batch after its append: per row the
    history pages (physical pool pages, INT8) and the exact pages (sidecar
    pages, logical order, the current page last), plus the token counts.
    Returns (old_indptr, old_indices, exact_indptr, exact_indices,
    exact_last_page_len, old_tokens, exact_tokens) as int32 arrays / lists."""
    o_ptr, e_ptr = [0], [0]
    o_idx, e_idx, last, o_tok, e_tok = [], [], [], [], []
    for row in batch.rows:
        st = row.expected_state
        part = partition(st.prompt_tokens, row.position + 1, policy)
        o_idx.extend(row.physical_pages[p] for p in part['history'])
        e_idx.extend(exact_slot(p, st.prompt_tokens, row.lease.slot, policy)
                     for p in part['exact'])
        o_ptr.append(len(o_idx))
        e_ptr.append(len(e_idx))
        last.append(row.position % PAGE + 1)
        o_tok.append(part['history_tokens'])
        e_tok.append(part['exact_tokens'])
    as32 = lambda x: np.asarray(x, dtype=np.int32)  # noqa: E731
    return as32(o_ptr), as32(o_idx), as32(e_ptr), as32(e_idx), as32(last), o_tok, e_tok


# ------------------------------------------------------------ GPU side
def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


class ServedPool:
    """A model's served PageGauge cache on one GPU: per layer one raw uint8
    pool allocation viewed as the four planes, the sidecars, prompt packing
    and the served decode step."""

    def __init__(self, layout: Layout, device="cuda", workspace_mb: int = 64,
                 warps_per_cta: int = 4):
        from .decode import PageGaugeDecode

        self.layout = layout
        self.device = torch.device(device)
        acc = layout.accounting()
        self.sidecars = allocate_sidecars(layout, device=self.device,
                                          cache_budget_bytes=acc['total_served_capacity_bytes'])
        per_layer = layout.physical_pages * acc['per_layer_page_bytes']
        self.raw = [torch.zeros(per_layer, dtype=torch.uint8, device=self.device)
                    for _ in range(layout.layers)]
        self.views = [dense_pool_views(r, layout.physical_pages, layout.kv_heads,
                                       layout.head_dim) for r in self.raw]
        self.decoder = PageGaugeDecode(torch.empty(workspace_mb << 20, dtype=torch.uint8,
                                                   device=self.device),
                                       warps_per_cta=warps_per_cta)
        self._batch = None

    # -------------------------------------------------------------- prefill
    def pack_prompt(self, layer: int, state: State, keys: torch.Tensor,
                    values: torch.Tensor) -> None:
        """Pack one request's prompt K/V (post-RoPE FP16 [T, Hkv, 128]) of one
        layer: centres = FP16 of the FP32 prompt mean (build_caches,
        scripts/benchmark_page_gauge_transformer.py:1199-1214), every complete
        prompt page bulk-quantised into its physical pool page, and the
        centred FP16 exact pages (prefix, suffix, tail) into the sidecar."""
        from .quantize import quantize_pages_into

        lay = self.layout
        T = state.prompt_tokens
        H, D = lay.kv_heads, lay.head_dim
        if tuple(keys.shape) != (T, H, D) or keys.shape != values.shape:
            raise ValueError(f'prompt K/V must be [{T},{H},{D}]')
        if keys.dtype != torch.float16 or values.dtype != torch.float16:
            raise ValueError('prompt K/V must be float16')
        slot = state.lease.slot
        sc = self.sidecars
        ck = keys.float().mean(0).half()
        cv = values.float().mean(0).half()
        sc['key_center'][layer, slot] = ck
        sc['value_center'][layer, slot] = cv
        sc['output_center'][layer, slot] = cv.repeat_interleave(lay.query_heads // H, dim=0)
        pages = -(-T // PAGE)
        padded_k = torch.zeros(pages * PAGE, H, D, dtype=torch.float16, device=keys.device)
        padded_v = torch.zeros_like(padded_k)
        padded_k[:T] = keys
        padded_v[:T] = values
        pk = padded_k.view(pages, PAGE, H, D)
        pv = padded_v.view(pages, PAGE, H, D)
        complete = T // PAGE
        v = self.views[layer]
        if complete:
            codes_k = torch.empty(complete, PAGE, H, D, dtype=torch.int8, device=keys.device)
            codes_v = torch.empty_like(codes_k)
            sk = torch.empty(complete, H, dtype=torch.float16, device=keys.device)
            sv = torch.empty_like(sk)
            quantize_pages_into(pk[:complete].contiguous(), pv[:complete].contiguous(), ck, cv,
                                codes_k, codes_v, sk, sv, 0, 'half_away')
            dst = torch.tensor(state.physical_pages[:complete], dtype=torch.long,
                               device=keys.device)
            v['key_codes'].index_copy_(0, dst, codes_k)
            v['value_codes'].index_copy_(0, dst, codes_v)
            v['key_scales'].index_copy_(0, dst, sk)
            v['value_scales'].index_copy_(0, dst, sv)
        part = partition(T, T, lay.policy)
        exact = list(part['exact'])
        slots = torch.tensor([exact_slot(p, T, slot, lay.policy) for p in exact],
                             dtype=torch.long, device=keys.device)
        src = torch.tensor(exact, dtype=torch.long, device=keys.device)
        ek = (pk.index_select(0, src).float() - ck.float()).half()
        ev = (pv.index_select(0, src).float() - cv.float()).half()
        # The padding rows of a partial last page stay zero in the ring.
        if T % PAGE:
            last = exact.index(pages - 1)
            ek[last, T % PAGE:] = 0
            ev[last, T % PAGE:] = 0
        sc['exact_key'][layer].index_copy_(0, slots, ek)
        sc['exact_value'][layer].index_copy_(0, slots, ev)

    # --------------------------------------------------------------- decode
    def plan(self, batch: DecodeBatch, old_split_pages: int = 0,
             exact_split_pages: int = 0) -> None:
        """Host planning of one decode step (outside CUDA-graph capture): the
        batch's device columns and page tables, shared by every layer."""
        lay = self.layout
        cols = batch.columns()
        dev = self.device
        as_dev = lambda x: torch.tensor(x, dtype=torch.int32).to(dev)  # noqa: E731
        self.positions = as_dev(cols['positions'])
        self.token_slots = as_dev(cols['physical_token_slots'])
        self.exact_slots = as_dev(cols['exact_token_slots'])
        self.center_rows = as_dev(cols['request_slots'])
        o_ptr, o_idx, e_ptr, e_idx, last, o_tok, e_tok = decode_tables(batch, lay.policy)
        self.old_tokens, self.exact_tokens = o_tok, e_tok
        self.tables = (o_ptr, o_idx, e_ptr, e_idx, last)
        self._old_indices = torch.from_numpy(o_idx).to(dev)
        self._exact_indices = torch.from_numpy(e_idx).to(dev)
        self._exact_last = torch.from_numpy(last).to(dev)
        self.decoder.plan(o_ptr, self._old_indices, e_ptr, self._exact_indices, self._exact_last,
                          lay.query_heads, lay.kv_heads, old_split_pages=old_split_pages,
                          exact_split_pages=exact_split_pages)
        B = len(batch.rows)
        self.center_out = torch.empty(B, lay.kv_heads, lay.head_dim, dtype=torch.float16,
                                      device=dev)
        self._batch = batch

    def step(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
             cos: torch.Tensor, sin: torch.Tensor, rotated_q: torch.Tensor,
             out: torch.Tensor | None = None, lse: torch.Tensor | None = None) -> torch.Tensor:
        """One layer of the planned decode step: q [B, Hq, 128], k / v
        [B, Hkv, 128] (row strides free), cos / sin [positions, 128] FP16.
        Appends the token at each row's position (RoPE, centring, page close
        into the pool) and returns the attention output [B, Hq, 128]."""
        if self._batch is None:
            raise RuntimeError('plan() must be called before step()')
        lay = self.layout
        B = len(self._batch.rows)
        for name, t, heads in (('q', q, lay.query_heads), ('k', k, lay.kv_heads),
                               ('v', v, lay.kv_heads), ('rotated_q', rotated_q, lay.query_heads)):
            if (t.dtype != torch.float16 or t.dim() != 3 or tuple(t.shape) != (B, heads, lay.head_dim)
                    or t.stride(2) != 1 or t.stride(1) != lay.head_dim):
                raise ValueError(f'{name} must be float16 [{B},{heads},{lay.head_dim}] with '
                                 f'contiguous heads')
        if rotated_q.stride(0) != lay.query_heads * lay.head_dim:
            raise ValueError('rotated_q must be contiguous')
        if cos.shape != sin.shape or cos.dim() != 2 or cos.shape[1] != lay.head_dim:
            raise ValueError('cos/sin must be matching [positions, 128] tables')
        sc = self.sidecars
        pool = self.views[layer]
        ek, ev = sc['exact_key'][layer], sc['exact_value'][layer]
        kc, vc = sc['key_center'][layer], sc['value_center'][layer]
        _lib.call('pg_rope_append_page_gauge_served', q.data_ptr(), k.data_ptr(), v.data_ptr(),
                  cos.data_ptr(), sin.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                  rotated_q.data_ptr(), ek.data_ptr(), ev.data_ptr(),
                  pool['key_codes'].data_ptr(), pool['value_codes'].data_ptr(),
                  pool['key_scales'].data_ptr(), pool['value_scales'].data_ptr(),
                  self.center_out.data_ptr(), q.stride(0), k.stride(0), v.stride(0), B,
                  lay.query_heads, lay.kv_heads, lay.physical_pages, ek.shape[0], kc.shape[0],
                  self.positions.data_ptr(), self.token_slots.data_ptr(),
                  self.exact_slots.data_ptr(), self.center_rows.data_ptr(), cos.stride(0),
                  cos.shape[0], _stream(q))
        # A one-page tail ring makes the page closed by this append INT8 at
        # the next step: that decode must wait for the append to complete.
        return self.decoder.run(rotated_q, pool['key_codes'], pool['value_codes'],
                                pool['key_scales'], pool['value_scales'], ek, ev,
                                self.center_out, out=out, lse=lse,
                                int8_after_wait=self.layout.policy.tail_pages == 1)
