"""Order matching engine: CPU reference book and the batched CUDA engine."""
from .book import (EngineConfig, OrderBook, init_msgs_from_l2, book_from_l2, MAXINT, INITID,
                   IOC, LIM, MKT, STRICT_BY_ID, INCLUDE_INITS, CANCEL_UNIFORM,
                   CANCEL_UNIFORM_AND_LARGE)
