"""CPU oracle for the vlak hot path -- TEST INFRASTRUCTURE ONLY.

A restatement, in numpy float64, of what the reference computes for
``vlak::softmax`` and the GQA fused attention, used as the checker in
``tests/``, in ``__graft_entry__.smoke()`` and as the timed CPU baseline of
``bench.py --impl reference``. Nothing in the product (the ``kernels``
package, the native libraries) imports or calls it.

Pinning: ``tests/test_oracle_golden.py`` checks these functions against
fixtures in ``tests/golden/`` that ``tests/golden/make_golden.py`` produced by
running the reference's own oracles (``ref_attn``, ``_analytic_params``,
``torch.softmax``) and real-mask fixture in the build container.
"""
from .softmax_oracle import softmax_rows, softmax_rows_torch_cpu  # noqa: F401
from .attention_oracle import (  # noqa: F401
    analytic_visible,
    gqa_attention,
    gqa_attention_torch_cpu,
    gqa_attention_varlen,
    masked_attention,
    sdpa_bhmd,
    solve_analytic_params,
    varlen_visible,
)
