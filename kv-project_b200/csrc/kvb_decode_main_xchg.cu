// kvb_decode_main_xchg.cu - instantiations of the sequence-split decode kernel (kvb_decode_xchg):
// the KIVI shapes with d_code 128 and at most two value groups per token.
#include "kvb_decode_inst.cuh"

KVB_INSTANTIATE_MAIN_XC(128, 4, 1, 1, kvb::KM_CHANNEL, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN_XC(128, 8, 1, 1, kvb::KM_CHANNEL, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN_XC(128, 4, 2, 2, kvb::KM_TOKEN, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN_XC(128, 8, 2, 2, kvb::KM_TOKEN, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN_XC(128, 4, 1, 1, kvb::KM_TOKEN, kvb::KV_ASYM)
KVB_INSTANTIATE_MAIN_XC(128, 8, 1, 1, kvb::KM_TOKEN, kvb::KV_ASYM)

KVB_STATUS_WORDS(status_words_main_xchg)
