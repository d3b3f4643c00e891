"""PageGauge-B200: the INT8 page-affine paged decode path on sm_100a.

Host code is Python/PyTorch (plumbing: tensors, streams, torch.distributed);
the work is done by hand-written CUDA kernels in libpagegauge_b200.so,
reached through the C ABI declared in include/pagegauge_b200.h.

Public surface (mirrors the reference's operator surface):
  runtime.load_append_extension()     fused RoPE/append/finalise + tail merge
  wrapper.make_page_gauge_wrapper()   INT8 page-affine decode plan/run
  wrapper.BatchDecodeWithPagedKVCacheWrapper   FP16 paged decode plan/run
  wrapper.merge_state_in_place()      base-2 LSE state merge
  decode.PageGaugeDecode              fused old-INT8 + exact-FP16 + merge + c_V
  heterogeneous.run_decode()          the single-page-table ABI
  quantize.quantize_page_gauge() / quantize_completed_kv_pages()
  quantize.quantize_pages()           the affine_group16 representation
  page_table.*                        request-major page-table helpers
  serving.*                           paged serving pool (vLLM-side layout)
  decoder.PageGaugeDecoder            Mistral-shaped decoder on these kernels
  scheduler.lookup()                  measured pages per work item
  shard.plan_shards()                 request or KV-head shards per GPU
"""

__version__ = "0.1.0"
