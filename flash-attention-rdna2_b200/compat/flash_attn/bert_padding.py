"""flash_attn.bert_padding -> fable_attn.bert_padding."""
from fable_attn.bert_padding import *  # noqa: F401,F403
from fable_attn.bert_padding import pad_input, unpad_input  # noqa: F401
