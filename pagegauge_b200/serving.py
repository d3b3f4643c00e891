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

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

PAGE = 16


# ----------------------------------------------------------------- policy
@dataclass(frozen=True)
class Policy:
    """Exact-page policy of a served request: ``prefix_pages`` pages from
    the start of the context, the ``suffix_pages`` pages that close the
    prompt, and a ring over the last ``tail_pages`` pages stay FP16; the
    rest of the completed pages are read as INT8 (partition.py:7-18)."""
    prefix_pages: int = 4
    suffix_pages: int = 128
    tail_pages: int = 48

    def __post_init__(self):
        counts = (self.prefix_pages, self.suffix_pages, self.tail_pages)
        if not all(type(c) is int for c in counts) or min(counts) < 0 or self.tail_pages == 0:
            raise ValueError('Invalid page policy')

    @property
    def storage_pages(self) -> int:
        """Sidecar pages one lease holds: prefix, suffix, then the ring."""
        return self.prefix_pages + self.suffix_pages + self.tail_pages

    def regions(self, prompt_pages: int, pages: int) -> tuple:
        """The three exact regions as half-open [begin, end) page ranges
        (prefix, prompt suffix, tail), in that order."""
        return ((0, self.prefix_pages), (prompt_pages - self.suffix_pages, prompt_pages),
                (pages - self.tail_pages, pages))

    def ring_base(self) -> int:
        return self.prefix_pages + self.suffix_pages


def _covered(runs) -> list:
    """Union of half-open page ranges as sorted, disjoint ranges."""
    out: list = []
    for b, e in sorted(r for r in runs if r[0] < r[1]):
        if out and b <= out[-1][1]:
            out[-1] = (out[-1][0], max(out[-1][1], e))
        else:
            out.append((b, e))
    return out


def partition(prompt_tokens, current_tokens, policy: Policy = Policy()) -> dict:
    """Split the logical pages of a request at ``current_tokens`` tokens into
    its exact pages (prefix, prompt suffix, tail) and its history pages,
    read as INT8 (partition.py:21-40).  The partial last page is always in
    the tail.  Returns the regions, the exact and history page tuples and
    the token counts of each side."""
    if (type(prompt_tokens) is not int or type(current_tokens) is not int
            or prompt_tokens <= 0 or current_tokens < prompt_tokens):
        raise ValueError('Invalid prompt/current length')
    prompt_pages = prompt_tokens // PAGE
    pages = -(-current_tokens // PAGE)
    # The prefix and suffix need a prompt that holds them, and at least one
    # page must lie between the prefix and the tail.
    if (prompt_pages < policy.prefix_pages + policy.suffix_pages
            or pages - policy.tail_pages <= policy.prefix_pages):
        raise ValueError('Prompt cannot support this policy; explicit FP16 fallback required')
    prefix, suffix, tail = (tuple(range(b, e)) for b, e in policy.regions(prompt_pages, pages))
    exact_runs = _covered(policy.regions(prompt_pages, pages))
    exact, history, cursor = [], [], 0
    for b, e in exact_runs:
        history.extend(range(cursor, b))
        exact.extend(range(b, e))
        cursor = e
    history.extend(range(cursor, pages))
    if not history or history[-1] == pages - 1:
        raise ValueError('No historical page or partial last page incorrectly quantized')
    return {'prefix': prefix, 'suffix': suffix, 'tail': tail,
            'exact': tuple(exact), 'history': tuple(history),
            'history_tokens': PAGE * len(history),
            'exact_tokens': current_tokens - PAGE * len(history),
            'tail_tokens': current_tokens - PAGE * (pages - policy.tail_pages)}


def exact_slot(logical_page, prompt_tokens, lease_slot, policy: Policy = Policy()) -> int:
    """Sidecar page of an exact logical page: the lease's block of
    ``storage_pages`` sidecar pages holds the prefix pages, then the prompt
    suffix pages, then the ring slot ``page % tail_pages``
    (partition.py:43-52)."""
    if logical_page < 0 or lease_slot < 0:
        raise ValueError('Negative page/lease slot')
    prompt_pages = prompt_tokens // PAGE
    suffix_begin = prompt_pages - policy.suffix_pages
    if logical_page < policy.prefix_pages:
        within = logical_page
    elif suffix_begin <= logical_page < prompt_pages:
        within = policy.prefix_pages + (logical_page - suffix_begin)
    else:
        within = policy.ring_base() + logical_page % policy.tail_pages
    return lease_slot * policy.storage_pages + within


def _aging(policy: Policy, prompt_tokens: int, tokens: int) -> tuple:
    """History pages gained when a request grows from ``tokens`` to
    ``tokens + 1`` tokens: when the new token opens a page, the ring's
    oldest page leaves the tail, and it turns INT8 unless the prefix or the
    prompt suffix keeps it exact."""
    if tokens % PAGE:
        return ()
    leaving = tokens // PAGE - policy.tail_pages  # the ring now starts one page later
    if leaving < 0:
        return ()
    (p0, p1), (s0, s1), _ = policy.regions(prompt_tokens // PAGE, tokens // PAGE + 1)
    return () if p0 <= leaving < p1 or s0 <= leaving < s1 else (leaving,)


# ---------------------------------------------------------------- layout
@dataclass(frozen=True)
class Layout:
    """Geometry of a served cache -- the persistent code pool (per layer:
    K/V codes and K/V page scales of ``physical_pages`` pages) and the
    per-lease sidecars (exact pages, key/value/output centres) of
    ``maximum_requests`` admissible requests -- and its byte accounting
    (cache_layout.py:6-38)."""
    layers: int
    physical_pages: int
    maximum_requests: int
    kv_heads: int = 8
    query_heads: int = 32
    head_dim: int = 128
    policy: Policy = Policy()

    def __post_init__(self):
        dims = (self.layers, self.physical_pages, self.maximum_requests, self.kv_heads,
                self.query_heads, self.head_dim)
        if not all(type(d) is int and d >= 1 for d in dims) or self.query_heads % self.kv_heads:
            raise ValueError('Invalid cache geometry')

    def planes(self) -> dict:
        """name -> (shape, bytes per element) of every served tensor; the
        first four form the pool, the rest the sidecars."""
        L, N, R = self.layers, self.physical_pages, self.maximum_requests
        H, Q, D = self.kv_heads, self.query_heads, self.head_dim
        exact = (L, R * self.policy.storage_pages, PAGE, H, D)
        return {'key_codes': ((L, N, PAGE, H, D), 1), 'value_codes': ((L, N, PAGE, H, D), 1),
                'key_scales': ((L, N, H), 2), 'value_scales': ((L, N, H), 2),
                'exact_key': (exact, 2), 'exact_value': (exact, 2),
                'key_center': ((L, R, H, D), 2), 'value_center': ((L, R, H, D), 2),
                'output_center': ((L, R, Q, D), 2)}

    def accounting(self) -> dict:
        sizes = {name: math.prod(shape) * width for name, (shape, width) in self.planes().items()}
        pool = sum(sizes[n] for n in POOL_PLANES)
        total = sum(sizes.values())
        return {'tensors': sizes, 'page_pool_bytes': pool,
                'reserved_sidecar_bytes': total - pool,
                'total_served_capacity_bytes': total,
                'per_layer_page_bytes': 2 * PAGE * self.kv_heads * self.head_dim
                                        + 2 * 2 * self.kv_heads,
                'scope': 'code pool planes plus the sidecars of every admissible lease, used '
                         'or not; model weights, decode workspace, CUDA graph pools, batch '
                         'buffers and allocator slack are budgeted separately'}

    def admissible_pages(self, cache_budget_bytes) -> int:
        """Pool pages a cache-only byte budget holds once every lease's
        sidecars are reserved (cache_layout.py:33-38)."""
        acc = self.accounting()
        left = cache_budget_bytes - acc['reserved_sidecar_bytes']
        if left < 0:
            raise MemoryError('Budget cannot hold reserved exact/center sidecars')
        return left // (self.layers * acc['per_layer_page_bytes'])

    @classmethod
    def for_budget(cls, layers: int, maximum_requests: int, cache_budget_bytes: int,
                   **kw) -> "Layout":
        """The largest pool a cache-only budget admits (e.g. a B200's HBM
        minus weights, workspace and graph pools)."""
        pages = cls(layers, 1, maximum_requests, **kw).admissible_pages(cache_budget_bytes)
        if pages < 1:
            raise MemoryError('Budget cannot hold reserved exact/center sidecars')
        return cls(layers, int(pages), maximum_requests, **kw)


POOL_PLANES = ('key_codes', 'value_codes', 'key_scales', 'value_scales')


# ----------------------------------------------------------------- views
def dense_pool_views(raw: torch.Tensor, physical_pages, kv_heads, head_dim=128) -> dict:
    """One layer's raw uint8 pool allocation as the four planes the kernels
    read -- K codes, V codes [pages, 16, Hkv, D] int8, K scales, V scales
    [pages, Hkv] fp16 -- back to back, no copy (cache_views.py:9-24)."""
    if not all(type(x) is int and x >= 1 for x in (physical_pages, kv_heads, head_dim)):
        raise ValueError('Positive integer pool geometry required')
    specs = (('key_codes', torch.int8, (physical_pages, PAGE, kv_heads, head_dim)),
             ('value_codes', torch.int8, (physical_pages, PAGE, kv_heads, head_dim)),
             ('key_scales', torch.float16, (physical_pages, kv_heads)),
             ('value_scales', torch.float16, (physical_pages, kv_heads)))
    widths = [math.prod(shape) * torch.empty(0, dtype=dt).element_size() for _, dt, shape in specs]
    if (raw.dtype != torch.uint8 or raw.ndim != 1 or not raw.is_contiguous()
            or raw.numel() != sum(widths) or raw.data_ptr() % 16):
        raise ValueError('Aligned contiguous uint8 layer allocation of exact size required')
    views, at = {}, 0
    for (name, dt, shape), width in zip(specs, widths):
        views[name] = raw[at:at + width].view(dt).view(shape)
        at += width
    return views


def from_engine_layer(layer: torch.Tensor, physical_pages, kv_heads) -> dict:
    """An engine's packed layer [pages, Hkv, 1, 2*16*128+4] uint8 read as
    the same four planes, without a copy (cache_views.py:27-39)."""
    if (layer.dtype != torch.uint8 or not layer.is_contiguous()
            or tuple(layer.shape) != (physical_pages, kv_heads, 1, 2 * PAGE * 128 + 4)):
        raise ValueError('Compact packed engine layer required; copying is forbidden')
    return dense_pool_views(layer.view(-1), physical_pages, kv_heads)


def zero_physical_pages(views: dict, page_ids) -> None:
    """Zero the given pool pages in all four planes, one kernel launch on
    the current stream (cache_views.py:42-62)."""
    planes = [views[n] for n in POOL_PLANES]
    count = planes[0].shape[0]
    pages = tuple(page_ids)
    consistent = all(t.device == planes[0].device and t.shape[0] == count for t in planes)
    valid = all(type(p) is int and 0 <= p < count for p in pages) and len(set(pages)) == len(pages)
    if not (consistent and valid):
        raise ValueError('Invalid physical pages or inconsistent pool views')
    if not pages:
        return
    if not planes[0].is_cuda:
        raise ValueError('pool views must be CUDA tensors')
    ids = torch.tensor(pages, dtype=torch.int32).to(planes[0].device, non_blocking=True)
    _lib.call('pg_zero_pool_pages', *(t.data_ptr() for t in planes), count,
              planes[0].shape[2], ids.data_ptr(), len(pages),
              torch.cuda.current_stream(planes[0].device).cuda_stream)


def allocate_sidecars(layout: Layout, *, device, cache_budget_bytes) -> dict:
    """Zeroed sidecar tensors for every admissible lease, shaped by the
    layout's plane table (sidecars.py:10-35)."""
    if type(cache_budget_bytes) is not int or cache_budget_bytes < 0:
        raise ValueError('Nonnegative integer cache-only byte budget required')
    if layout.accounting()['total_served_capacity_bytes'] > cache_budget_bytes:
        raise MemoryError('Code pool plus all reserved sidecars exceed cache budget')
    return {name: torch.zeros(shape, dtype=torch.float16, device=device)
            for name, (shape, _) in layout.planes().items() if name not in POOL_PLANES}


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


def _block_table(physical_pages, count: int) -> tuple:
    """A request's physical pages: exactly ``count`` distinct non-negative
    integers."""
    pages = tuple(physical_pages)
    if (len(pages) != count or len(set(pages)) != count
            or not all(type(p) is int and p >= 0 for p in pages)):
        raise ValueError('Wrong/duplicate physical block table')
    return pages


class RequestSlots:
    """Admission control of the served cache: ``maximum_requests`` sidecar
    slots, each lent to one live request at a time under a generation
    count, and the ownership of every physical pool page a live request
    holds (request_slots.py:20-93).  Slots are handed out lowest first."""

    def __init__(self, maximum_requests, policy: Policy = Policy()):
        if type(maximum_requests) is not int or maximum_requests < 1:
            raise ValueError('Positive fixed admission capacity required')
        self.policy = policy
        self._occupied = [False] * maximum_requests
        self.generations = [0] * maximum_requests
        self.states: dict[str, State] = {}
        self.page_owner: dict[int, Lease] = {}

    @property
    def free(self) -> list:
        """Slots no live request holds, ascending."""
        return [i for i, used in enumerate(self._occupied) if not used]

    def _claim(self, pages, lease: Lease) -> None:
        for p in pages:
            self.page_owner[p] = lease

    def admit(self, request_id, prompt_tokens, physical_pages) -> Lease:
        if not isinstance(request_id, str) or not request_id or request_id in self.states:
            raise ValueError('Invalid or duplicate live request ID')
        partition(prompt_tokens, prompt_tokens, self.policy)  # the policy must fit the prompt
        pages = _block_table(physical_pages, -(-prompt_tokens // PAGE))
        if any(p in self.page_owner for p in pages):
            raise ValueError('Cross-request page sharing is disabled')
        free = self.free
        if not free:
            raise MemoryError('Declared exact-sidecar admission capacity reached')
        slot = free[0]
        self._occupied[slot] = True
        self.generations[slot] += 1
        lease = Lease(request_id, slot, self.generations[slot])
        self.states[request_id] = State(lease, prompt_tokens, prompt_tokens, pages)
        self._claim(pages, lease)
        return lease

    def state(self, lease: Lease) -> State:
        current = self.states.get(lease.request_id)
        if current is None or current.lease != lease:
            raise ValueError('Stale request lease/center generation')
        return current

    def batch(self, request_ids) -> tuple:
        rows = tuple(request_ids)
        if len(set(rows)) != len(rows):
            raise ValueError('Duplicate batch row')
        missing = [r for r in rows if r not in self.states]
        if missing:
            raise ValueError('Unknown scheduled request')
        return tuple(self.states[r].lease for r in rows)

    def append(self, lease: Lease, position, physical_pages) -> dict:
        """Record the token at ``position`` (the request's next one) with the
        request's block table after it; returns the page it closes, the
        pages that turned INT8 and the new partition."""
        current = self.state(lease)
        if position != current.current_tokens:
            raise ValueError('Skipped/replayed token or wrong per-request position')
        tokens = position + 1
        pages = _block_table(physical_pages, -(-tokens // PAGE))
        held = len(current.physical_pages)
        if pages[:held] != current.physical_pages:
            raise ValueError('Preemption/remapping is not supported in phase one')
        if any(p in self.page_owner for p in pages[held:]):
            raise ValueError('New physical page belongs to a live request')
        after = partition(current.prompt_tokens, tokens, self.policy)
        aged = _aging(self.policy, current.prompt_tokens, position)
        if any(p >= tokens // PAGE for p in aged):
            raise ValueError('Attempt to consume an unfinished INT8 page')
        self._claim(pages[held:], lease)
        self.states[lease.request_id] = State(lease, current.prompt_tokens, tokens, pages)
        return {'lease': lease, 'position': position,
                'closed_page': position // PAGE if tokens % PAGE == 0 else None,
                'new_history_pages': aged, 'partition': after}

    def release(self, lease: Lease) -> None:
        current = self.state(lease)
        if any(self.page_owner.get(p) != lease for p in current.physical_pages):
            raise ValueError('Page ownership corrupted')
        for p in current.physical_pages:
            del self.page_owner[p]
        del self.states[lease.request_id]
        self._occupied[lease.slot] = False


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
        """The integer columns a device step consumes, one entry per row in
        scheduled order (decode_metadata.py:28-35)."""
        return {'request_slots': tuple(r.lease.slot for r in self.rows),
                'generations': tuple(r.lease.generation for r in self.rows),
                'positions': tuple(r.position for r in self.rows),
                'physical_token_slots': tuple(r.physical_token_slot for r in self.rows),
                'exact_token_slots': tuple(r.exact_token_slot for r in self.rows)}


def _decode_row(manager: RequestSlots, lease: Lease, position, physical_pages,
                taken: set) -> DecodeRow:
    """One row of a decode batch, validated against the manager without
    changing it; ``taken`` collects the physical pages the batch uses."""
    current = manager.state(lease)
    if type(position) is not int or position != current.current_tokens:
        raise ValueError('Wrong next token position')
    pages = _block_table(physical_pages, position // PAGE + 1)
    held = len(current.physical_pages)
    if pages[:held] != current.physical_pages:
        raise ValueError('Physical remapping is unsupported')
    if any(p in taken for p in pages[held:]):
        raise ValueError('Physical page alias across batch')
    taken.update(pages[held:])
    partition(current.prompt_tokens, position + 1, manager.policy)
    aged = _aging(manager.policy, current.prompt_tokens, position)
    if any(p >= (position + 1) // PAGE for p in aged):
        raise ValueError('Cannot quantize incomplete page')
    page, token = divmod(position, PAGE)
    slot_of = lambda lp: exact_slot(lp, current.prompt_tokens, lease.slot,  # noqa: E731
                                    manager.policy)
    return DecodeRow(lease, current, position, pages, pages[page] * PAGE + token,
                     slot_of(page) * PAGE + token, aged, tuple(pages[p] for p in aged),
                     tuple(slot_of(p) for p in aged))


def prepare_decode(manager: RequestSlots, scheduled) -> DecodeBatch:
    """Validate a batch of (lease, next position, full block table) rows and
    derive its device metadata, changing nothing in the manager
    (decode_metadata.py:38-62)."""
    seen, taken, rows = set(), set(manager.page_owner), []
    for lease, position, physical_pages in scheduled:
        manager.state(lease)
        if lease.request_id in seen:
            raise ValueError('Duplicate scheduled request')
        seen.add(lease.request_id)
        rows.append(_decode_row(manager, lease, position, physical_pages, taken))
    return DecodeBatch(tuple(rows))


def commit_decode(manager: RequestSlots, batch: DecodeBatch) -> tuple:
    """Advance the manager by a batch whose device work has completed.  Every
    row must still describe its request's current state and re-derive to
    the same metadata (decode_metadata.py:65-76)."""
    if any(manager.state(r.lease) != r.expected_state for r in batch.rows):
        raise ValueError('Decode batch is stale')
    taken = set(manager.page_owner)
    for row in batch.rows:
        if _decode_row(manager, row.lease, row.position, row.physical_pages, taken) != row:
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
