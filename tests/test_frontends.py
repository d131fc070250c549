"""Argument checks of the attention and normalisation front-ends (CPU, fake tensors).

Every invalid call raises the reference's exception type and message, in the reference's
order (src/radeon_kernels/ops/{sdpa,paged_attention,rms_norm,add_rms_norm}/api.py), before
anything is dispatched; valid calls produce the dispatch signature and native arguments
the manifests and pack entrypoints expect.
"""

from __future__ import annotations

import pytest

from fakes import FakeTensor, FakeTorch
from radeon_kernels.ops.add_rms_norm.api import _execute as arms
from radeon_kernels.ops.paged_attention.api import _execute as paged
from radeon_kernels.ops.rms_norm.api import _execute as rms
from radeon_kernels.ops.sdpa.api import _execute as sdpa


class Capture:
    def __init__(self):
        self.call = None

    def execute(self, **kw):
        self.call = kw
        return (1, 2)


def T(shape, **kw):
    return FakeTensor(shape, **kw)


cases = {
 "sdpa": [
  ("q rank", lambda: (T((1,2,8)), T((1,2,8,64)), T((1,2,8,64)))),
  ("k not tensor", lambda: (T((1,2,8,64)), "x", T((1,2,8,64)))),
  ("v dtype", lambda: (T((1,2,8,64)), T((1,2,8,64)), T((1,2,8,64), dtype="bfloat16"))),
  ("q float32", lambda: (T((1,2,8,64), dtype="float32"), T((1,2,8,64)), T((1,2,8,64)))),
  ("kv shape", lambda: (T((1,2,8,64)), T((1,2,8,64)), T((1,2,9,64)))),
  ("batch", lambda: (T((1,2,8,64)), T((2,2,8,64)), T((2,2,8,64)))),
  ("zero dim", lambda: (T((1,0,8,64)), T((1,2,8,64)), T((1,2,8,64)))),
  ("seq", lambda: (T((1,2,8,64)), T((1,2,9,64)), T((1,2,9,64)))),
  ("head_dim", lambda: (T((1,2,8,96)), T((1,2,8,96)), T((1,2,8,96)))),
  ("head_dim mismatch", lambda: (T((1,2,8,64)), T((1,2,8,128)), T((1,2,8,128)))),
  ("gqa", lambda: (T((1,3,8,64)), T((1,2,8,64)), T((1,2,8,64)))),
  ("noncontig", lambda: (T((1,2,8,64), contiguous=False), T((1,2,8,64)), T((1,2,8,64)))),
  ("grad", lambda: (T((1,2,8,64)), T((1,2,8,64), requires_grad=True), T((1,2,8,64)))),
 ],
 "paged": [
  ("q rank", lambda: (T((2,8)), T((4,16,2,128)), T((4,16,2,128)), T((2,2), dtype="int32"), T((2,), dtype="int32"))),
  ("kc rank", lambda: (T((2,8,128)), T((4,16,128)), T((4,16,2,128)), T((2,2), dtype="int32"), T((2,), dtype="int32"))),
  ("vc dtype", lambda: (T((2,8,128)), T((4,16,2,128)), T((4,16,2,128), dtype="bfloat16"), T((2,2), dtype="int32"), T((2,), dtype="int32"))),
  ("cache shape", lambda: (T((2,8,128)), T((4,16,2,128)), T((5,16,2,128)), T((2,2), dtype="int32"), T((2,), dtype="int32"))),
  ("bt float", lambda: (T((2,8,128)), T((4,16,2,128)), T((4,16,2,128)), T((2,2)), T((2,), dtype="int32"))),
  ("bt rank", lambda: (T((2,8,128)), T((4,16,2,128)), T((4,16,2,128)), T((2,), dtype="int32"), T((2,), dtype="int32"))),
  ("cl rank", lambda: (T((2,8,128)), T((4,16,2,128)), T((4,16,2,128)), T((2,2), dtype="int32"), T((2,1), dtype="int32"))),
  ("idx dtype mix", lambda: (T((2,8,128)), T((4,16,2,128)), T((4,16,2,128)), T((2,2), dtype="int32"), T((2,), dtype="int64"))),
  ("zero", lambda: (T((0,8,128)), T((4,16,2,128)), T((4,16,2,128)), T((0,2), dtype="int32"), T((0,), dtype="int32"))),
  ("head_dim", lambda: (T((2,8,80)), T((4,16,2,80)), T((4,16,2,80)), T((2,2), dtype="int32"), T((2,), dtype="int32"))),
  ("gqa", lambda: (T((2,10,128)), T((4,16,4,128)), T((4,16,4,128)), T((2,2), dtype="int32"), T((2,), dtype="int32"))),
  ("bt shape", lambda: (T((2,8,128)), T((4,16,2,128)), T((4,16,2,128)), T((3,2), dtype="int32"), T((2,), dtype="int32"))),
  ("bt zero", lambda: (T((2,8,128)), T((4,16,2,128)), T((4,16,2,128)), T((2,0), dtype="int32"), T((2,), dtype="int32"))),
  ("cl shape", lambda: (T((2,8,128)), T((4,16,2,128)), T((4,16,2,128)), T((2,2), dtype="int32"), T((3,), dtype="int32"))),
  ("noncontig", lambda: (T((2,8,128)), T((4,16,2,128), contiguous=False), T((4,16,2,128)), T((2,2), dtype="int32"), T((2,), dtype="int32"))),
  ("grad", lambda: (T((2,8,128), requires_grad=True), T((4,16,2,128)), T((4,16,2,128)), T((2,2), dtype="int32"), T((2,), dtype="int32"))),
 ],
 "rms": [
  ("x rank", lambda: (T((8,)), T((8,)), 1e-6)),
  ("w rank", lambda: (T((2,8)), T((8,1)), 1e-6)),
  ("w dtype", lambda: (T((2,8)), T((8,), dtype="bfloat16"), 1e-6)),
  ("hidden", lambda: (T((2,8)), T((4,)), 1e-6)),
  ("eps 0", lambda: (T((2,8)), T((8,)), 0)),
  ("eps bool", lambda: (T((2,8)), T((8,)), True)),
  ("eps str", lambda: (T((2,8)), T((8,)), "1e-6")),
  ("x f32", lambda: (T((2,8), dtype="float32"), T((8,), dtype="float32"), 1e-6)),
 ],
 "arms": [
  ("x rank", lambda: (T((8,)), T((2,8)), T((8,)), 1e-6)),
  ("r rank", lambda: (T((2,8)), T((8,)), T((8,)), 1e-6)),
  ("w rank", lambda: (T((2,8)), T((2,8)), T((2,8)), 1e-6)),
  ("r dtype", lambda: (T((2,8)), T((2,8), dtype="bfloat16"), T((8,)), 1e-6)),
  ("w dtype", lambda: (T((2,8)), T((2,8)), T((8,), dtype="bfloat16"), 1e-6)),
  ("shape", lambda: (T((2,8)), T((3,8)), T((8,)), 1e-6)),
  ("hidden", lambda: (T((2,8)), T((2,8)), T((4,)), 1e-6)),
  ("eps", lambda: (T((2,8)), T((2,8)), T((8,)), -1.0)),
 ],
}

OPS = {"sdpa": sdpa, "paged": paged, "rms": rms, "arms": arms}
EXPECTED = {'sdpa:q rank': ('ValueError', 'sdpa query must be rank 4'),
 'sdpa:k not tensor': ('TypeError', 'sdpa key must be a PyTorch tensor'),
 'sdpa:v dtype': ('TypeError', 'sdpa key and value must use the same dtype'),
 'sdpa:q float32': ('TypeError', 'sdpa supports torch.float16 and torch.bfloat16 tensors'),
 'sdpa:kv shape': ('ValueError', 'sdpa key and value must have the same shape'),
 'sdpa:batch': ('ValueError', 'sdpa query, key and value must share the batch dimension'),
 'sdpa:zero dim': ('ValueError', 'sdpa tensor dimensions must be positive'),
 'sdpa:seq': ('ValueError', 'sdpa 1.0 requires equal query and KV sequence lengths'),
 'sdpa:head_dim': ('ValueError', 'sdpa head_dim must match and be one of 64, 128, 256'),
 'sdpa:head_dim mismatch': ('ValueError', 'sdpa head_dim must match and be one of 64, 128, 256'),
 'sdpa:gqa': ('ValueError', 'sdpa query_heads must be divisible by kv_heads'),
 'sdpa:noncontig': ('ValueError', 'sdpa inputs must be contiguous'),
 'sdpa:grad': ('ValueError', 'sdpa is inference-only and does not support autograd'),
 'paged:q rank': ('ValueError', 'paged_attention_decode query must be rank 3'),
 'paged:kc rank': ('ValueError', 'paged_attention_decode key_cache must be rank 4'),
 'paged:vc dtype': ('TypeError', 'paged_attention_decode key_cache and value_cache must use the same dtype'),
 'paged:cache shape': ('ValueError',
                       'paged_attention_decode key_cache and value_cache must have the same shape'),
 'paged:bt float': ('TypeError', 'paged_attention_decode index tensors must use torch.int32 or torch.int64'),
 'paged:bt rank': ('ValueError', 'paged_attention_decode block_tables must be rank 2'),
 'paged:cl rank': ('ValueError', 'paged_attention_decode context_lengths must be rank 1'),
 'paged:idx dtype mix': ('TypeError',
                         'paged_attention_decode block_tables and context_lengths must use the same dtype'),
 'paged:zero': ('ValueError', 'paged_attention_decode tensor dimensions must be positive'),
 'paged:head_dim': ('ValueError',
                    'paged_attention_decode head_dim must match cache and be one of 64, 128, 256'),
 'paged:gqa': ('ValueError', 'paged_attention_decode query_heads must be divisible by kv_heads'),
 'paged:bt shape': ('ValueError', 'paged_attention_decode block_tables must have shape [batch, max_blocks]'),
 'paged:bt zero': ('ValueError', 'paged_attention_decode block_tables must have shape [batch, max_blocks]'),
 'paged:cl shape': ('ValueError',
                    'paged_attention_decode context_lengths must contain one length per sequence'),
 'paged:noncontig': ('ValueError', 'paged_attention_decode inputs must be contiguous'),
 'paged:grad': ('ValueError', 'paged_attention_decode is inference-only and does not support autograd'),
 'rms:x rank': ('ValueError', 'rms_norm x must be rank 2'),
 'rms:w rank': ('ValueError', 'rms_norm weight must be rank 1'),
 'rms:w dtype': ('TypeError', 'rms_norm x and weight must use the same dtype'),
 'rms:hidden': ('ValueError', 'rms_norm weight must match the hidden dimension'),
 'rms:eps 0': ('ValueError', 'rms_norm eps must be positive and finite'),
 'rms:eps bool': ('TypeError', 'rms_norm eps must be a number'),
 'rms:eps str': ('TypeError', 'rms_norm eps must be a number'),
 'rms:x f32': ('TypeError', 'rms_norm supports torch.float16 and torch.bfloat16 tensors'),
 'arms:x rank': ('ValueError', 'add_rms_norm x must be rank 2'),
 'arms:r rank': ('ValueError', 'add_rms_norm residual must be rank 2'),
 'arms:w rank': ('ValueError', 'add_rms_norm weight must be rank 1'),
 'arms:r dtype': ('TypeError', 'add_rms_norm x and residual must use the same dtype'),
 'arms:w dtype': ('TypeError', 'add_rms_norm x and weight must use the same dtype'),
 'arms:shape': ('ValueError', 'add_rms_norm x and residual must have the same shape'),
 'arms:hidden': ('ValueError', 'add_rms_norm weight must match the hidden dimension'),
 'arms:eps': ('ValueError', 'add_rms_norm eps must be positive and finite')}


@pytest.mark.parametrize("op, name", [(op, name) for op, cs in cases.items() for name, _ in cs])
def test_invalid_call_raises_before_dispatch(op, name):
    make = dict(cases[op])[name]
    runtime = Capture()
    kind, message = EXPECTED[f"{op}:{name}"]
    with pytest.raises(Exception) as caught:
        OPS[op](*make(), torch_module=FakeTorch(), runtime=runtime)
    assert (type(caught.value).__name__, str(caught.value)) == (kind, message)
    assert runtime.call is None

valid = {
 "sdpa": (T((2,8,64,128)), T((2,2,64,128)), T((2,2,64,128)), True, None),
 "sdpa2": (T((1,4,16,64), dtype="bfloat16"), T((1,4,16,64), dtype="bfloat16"), T((1,4,16,64), dtype="bfloat16"), False, 0.5),
 "paged": (T((2,8,128)), T((4,16,2,128)), T((4,16,2,128)), T((2,2), dtype="int32"), T((2,), dtype="int32"), None),
 "paged2": (T((3,32,256), dtype="bfloat16"), T((9,8,8,256), dtype="bfloat16"), T((9,8,8,256), dtype="bfloat16"), T((3,3), dtype="int64"), T((3,), dtype="int64"), 0.1),
 "rms": (T((5,8)), T((8,)), 1e-5),
 "arms": (T((5,8), dtype="bfloat16"), T((5,8), dtype="bfloat16"), T((8,), dtype="bfloat16"), 2),
}
FN = {"sdpa": sdpa, "sdpa2": sdpa, "paged": paged, "paged2": paged, "rms": rms, "arms": arms}
VALID = {'sdpa': {'operator': 'sdpa',
          'semver': '1.0',
          'signature': {'dtype': 'fp16',
                        'batch': 2,
                        'query_heads': 8,
                        'kv_heads': 2,
                        'sequence': 64,
                        'head_dim': 128,
                        'layout': 'batch_head_sequence_dim',
                        'attention_mode': 'causal',
                        'scale_mode': 'default',
                        'contiguous': True,
                        'requires_grad': False},
          'device': 0,
          'native': ['T(2, 8, 64, 128)',
                     'T(2, 2, 64, 128)',
                     'T(2, 2, 64, 128)',
                     'True',
                     '0.08838834764831843'],
          'fallback_selected': 'cuda/sdpa',
          'result': '(1, 2)'},
 'sdpa2': {'operator': 'sdpa',
           'semver': '1.0',
           'signature': {'dtype': 'bf16',
                         'batch': 1,
                         'query_heads': 4,
                         'kv_heads': 4,
                         'sequence': 16,
                         'head_dim': 64,
                         'layout': 'batch_head_sequence_dim',
                         'attention_mode': 'noncausal',
                         'scale_mode': 'explicit',
                         'contiguous': True,
                         'requires_grad': False},
           'device': 0,
           'native': ['T(1, 4, 16, 64)', 'T(1, 4, 16, 64)', 'T(1, 4, 16, 64)', 'False', '0.5'],
           'fallback_selected': 'cuda/sdpa',
           'result': '(1, 2)'},
 'paged': {'operator': 'paged_attention_decode',
           'semver': '1.0',
           'signature': {'dtype': 'fp16',
                         'batch': 2,
                         'query_heads': 8,
                         'kv_heads': 2,
                         'head_dim': 128,
                         'num_blocks': 4,
                         'block_size': 16,
                         'max_blocks_per_sequence': 2,
                         'index_dtype': 'int32',
                         'cache_layout': 'block_slot_head_dim',
                         'scale_mode': 'default',
                         'contiguous': True,
                         'requires_grad': False},
           'device': 0,
           'native': ['T(2, 8, 128)',
                      'T(4, 16, 2, 128)',
                      'T(4, 16, 2, 128)',
                      'T(2, 2)',
                      'T(2,)',
                      '0.08838834764831843'],
           'fallback_selected': 'cuda/paged_attention_decode',
           'result': '(1, 2)'},
 'paged2': {'operator': 'paged_attention_decode',
            'semver': '1.0',
            'signature': {'dtype': 'bf16',
                          'batch': 3,
                          'query_heads': 32,
                          'kv_heads': 8,
                          'head_dim': 256,
                          'num_blocks': 9,
                          'block_size': 8,
                          'max_blocks_per_sequence': 3,
                          'index_dtype': 'int64',
                          'cache_layout': 'block_slot_head_dim',
                          'scale_mode': 'explicit',
                          'contiguous': True,
                          'requires_grad': False},
            'device': 0,
            'native': ['T(3, 32, 256)', 'T(9, 8, 8, 256)', 'T(9, 8, 8, 256)', 'T(3, 3)', 'T(3,)', '0.1'],
            'fallback_selected': 'cuda/paged_attention_decode',
            'result': '(1, 2)'},
 'rms': {'operator': 'rms_norm',
         'semver': '1.0',
         'signature': {'dtype': 'fp16',
                       'tokens': 5,
                       'hidden': 8,
                       'eps': 1e-05,
                       'contiguous': True,
                       'requires_grad': False},
         'device': 0,
         'native': ['T(5, 8)', 'T(8,)', '1e-05'],
         'fallback_selected': 'cuda/rms_norm',
         'result': '(1, 2)'},
 'arms': {'operator': 'add_rms_norm',
          'semver': '1.0',
          'signature': {'dtype': 'bf16',
                        'tokens': 5,
                        'hidden': 8,
                        'eps': 2.0,
                        'contiguous': True,
                        'requires_grad': False},
          'device': 0,
          'native': ['T(5, 8)', 'T(5, 8)', 'T(8,)', '2.0'],
          'fallback_selected': 'cuda/add_rms_norm',
          'result': '(1, 2)'}}


@pytest.mark.parametrize("name", sorted(VALID))
def test_valid_call_signature_and_native_arguments(name):
    runtime = Capture()
    result = FN[name](*valid[name], torch_module=FakeTorch(), runtime=runtime)
    c = runtime.call
    got = {"operator": c["operator"], "semver": c["semantic_version"], "signature": c["signature"], "device": c["device_index"],
           "native": [repr(a) if not hasattr(a, "shape") else f"T{a.shape}" for a in c["native_arguments"]],
           "fallback_selected": c["fallback_selected"], "result": repr(result)}
    assert got == VALID[name]
