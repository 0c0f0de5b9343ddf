"""CPU oracle for the inferd decode hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's algorithms (likhith-v1/inferd), used as the
checker for the CUDA kernels in inferd_b200:

* paged gather + single-query GQA attention   core/paged_attn.py:20-167
* the KV append write of PagedKVCache          core/paged_cache.py:151-189
* causal multi-query (speculative verify) attention, following the HF eager path the
  reference's verify forward runs (core/spec_decode.py:135 ->
  transformers.models.qwen3_5.modeling_qwen3_5.eager_attention_forward)
* per-output-channel e4m3 weight quantisation and dequant-then-matmul (torchao 0.17.0
  Float8WeightOnlyConfig as configured in bench/model_loader.py:46-58; torchao is not
  vendored, so the published per-channel absmax/448 recipe is restated)
* decode-step sampling: temperature + top-p nucleus probabilities and the inverse-CDF
  draw                                          core/spec_decode.py:14-35

Parity pins: tests/golden/*.npz hold outputs of the reference itself (imported from its
source tree by tests/golden/make_golden.py) and of torch's float8_e4m3fn cast; the
oracle is checked against every one of them by tests/test_oracle_golden.py.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this
package, and only as the checker or the timed CPU baseline.  The product path
(inferd_b200) never imports it.
"""

from .paged import (  # noqa: F401
    batched_paged_attention,
    dense_attention,
    gather_paged_kv,
    paged_attention,
    reshape_and_cache,
    sdpa_attention,
    verify_attention,
)
from .fp8 import (  # noqa: F401
    E4M3_MAX,
    e4m3_decode,
    e4m3_encode,
    fp8_dynamic_linear,
    fp8_linear,
    quantize_dynamic,
    quantize_per_channel,
)
from .sampling import (  # noqa: F401
    accept_resample,
    kept_mask_fixed,
    nucleus_probs,
    philox4x32_10,
    row_random64,
    row_uniform,
    sample_fixed,
    to_fixed,
    weight_scale,
)
