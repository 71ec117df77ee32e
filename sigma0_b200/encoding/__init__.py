"""Message encodings (1/22/23/24/26 tokens per message)."""
from .tokenizer import (MASK_TOK, HIDDEN_TOK, NA_TOK, START_TOK, NA_VAL, MASK_VAL,
                        HIDDEN_VAL, START_VAL, RAW_FIELDS, MODES, MessageTokenizer,
                        get_tokenizer)
from .selector import (SUPPORTED_TOKEN_MODES, DEFAULT_TOKEN_MODE, Message_Tokenizer, Vocab,
                       set_token_mode, get_token_mode, supported_token_modes,
                       encode_msgs, decode_msgs, active_tokenizer)
