// kvb_decode_main_token.cu - decode_main instantiations: KIVI per-token keys.
#include "kvb_decode_inst.cuh"

KVB_INSTANTIATE_MAIN(128, 4, 2, 2, kvb::KM_TOKEN, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN(128, 8, 2, 2, kvb::KM_TOKEN, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN(128, 4, 1, 1, kvb::KM_TOKEN, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN(128, 8, 1, 1, kvb::KM_TOKEN, kvb::KV_ASYM)

KVB_STATUS_WORDS(status_words_main_token)
