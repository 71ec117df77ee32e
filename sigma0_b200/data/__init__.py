"""Data: synthetic order flow, book transform, windowed datasets."""
from .synthetic import generate_day, make_sequences, SyntheticDay
from .book_transform import transform_l2_numpy, transform_books_numpy, transform_books_torch
from .dataset import LobWindowDataset, collate
