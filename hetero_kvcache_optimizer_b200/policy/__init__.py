from .prefetcher import AsyncPrefetcher, PagePrefetcher
