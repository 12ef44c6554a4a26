"""CPU oracle for SlimKV's decode-time latent attention path.

TEST INFRASTRUCTURE ONLY.  This package restates, in plain numpy, the
algorithms of the reference implementation (Strandding/SlimKV) on the hot
path: eager grouped attention, BF16-exact RoPE, the LSE merge, query
absorption and value up-projection, the decode-step Beacon schedule, the
prefill interleave rule, the prefill window projection / RoPE / cache
append and the paged-cache addressing.  Each function cites
the reference file and line range it follows.

It is the parity checker for the CUDA path and the timed CPU baseline.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and
``--impl reference`` legs may import it.  The product package
``slimkv_b200`` never imports, links or calls anything in here.

The restatement is pinned against golden vectors produced by running the
reference's own Python code (``tests/golden/make_golden.py``).
"""
from .bf16 import round_bf16, bf16_bits, from_bf16_bits
from .attention import eager_attention, merge_attention, project_query, project_value
from .rope import rope_bf16, rope_tables, raw_key_positions
from .decode import latent_decode_attention
from .schedule import FastDecodeSchedule, interleave_roles, paged_restore_roles
from .pages import BeaconPageLayout, beacon_page_slots, raw_page_slots, beacon_block_size
from .splits import latent_splits, dense_splits, original_splits
from .prefill import prefill_metadata, project_with_beacon, prefill_rope, flush_chunk
from .reconstruct import materialize, reconstruct_decode_attention
