"""CPU oracle for the paged-KV attention path (numpy restatement of vllm-rlt).

TEST INFRASTRUCTURE. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` (``cpu_baseline`` and ``--impl reference``) may
import this package, and only as the checker or the timed CPU reference --
never as the thing measured for the GPU path or shipped in the product. The
``vllm_rlt_b200`` package never imports it.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
golden vectors produced by the reference itself (``tests/golden/make_golden.py``
imports the reference package and runs its torch code and, through Triton's
CPU interpreter, its Triton kernels).
"""

from .ref_ops import (  # noqa: F401
    bf16_to_f32,
    expand_prefill,
    f32_to_bf16,
    finalize,
    finalize_token,
    from_f32,
    gather,
    kv_write,
    metadata,
    paged_attention,
    paged_prefill,
    prepare_rows,
    scatter,
    stage_prefill,
    to_f32,
)
