// kvb_decode_main_midrise.cu - decode_main instantiations: mid-rise (STRATA / spectral) codes.
#include "kvb_decode_inst.cuh"

KVB_INSTANTIATE_MAIN(128, 4, 1, 1, kvb::KM_TOKEN, kvb::KV_MIDRISE)
KVB_INSTANTIATE_MAIN(128, 8, 1, 1, kvb::KM_TOKEN, kvb::KV_MIDRISE)
KVB_INSTANTIATE_MAIN(64, 4, 1, 1, kvb::KM_TOKEN, kvb::KV_MIDRISE)
KVB_INSTANTIATE_MAIN(32, 4, 1, 1, kvb::KM_TOKEN, kvb::KV_MIDRISE)
KVB_INSTANTIATE_MAIN(32, 8, 1, 1, kvb::KM_TOKEN, kvb::KV_MIDRISE)

KVB_STATUS_WORDS(status_words_main_midrise)
