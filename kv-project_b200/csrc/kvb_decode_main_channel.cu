// kvb_decode_main_channel.cu - decode_main instantiations: KIVI per-channel keys.
#include "kvb_decode_inst.cuh"

KVB_INSTANTIATE_MAIN(128, 4, 1, 4, kvb::KM_CHANNEL, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN(128, 4, 1, 2, kvb::KM_CHANNEL, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN(128, 4, 1, 1, kvb::KM_CHANNEL, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN(128, 8, 1, 1, kvb::KM_CHANNEL, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN(128, 8, 1, 2, kvb::KM_CHANNEL, kvb::KV_ASYM)

KVB_STATUS_WORDS(status_words_main_channel)
