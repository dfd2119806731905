"""ORACLE — test infrastructure only.

A CPU restatement of the reference's expert hot path (codec, on-disk format,
router / permute / expert FFN / combine).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import anything
here, and only as the checker or the timed CPU baseline; the product under
``zipmoe-icml26_b200/`` never imports, links or runs it.

Pinning: the LZ4 restatement (``lz4_block.c``) is checked byte for byte against
liblz4 (the reference's codec library, 1.9.4 in this image) on every fixture;
the MoE-block restatement is checked against fixtures produced by running the
reference's own ``customized/qwen.py`` and ``customized/deepseek.py`` blocks
(``tests/golden/make_golden.py``).  The Switch router comes from
transformers<4.47, which is not installed: that part is unpinned.
"""
