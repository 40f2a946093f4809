// GPU drafter (placeholder).
extern "C" int lng_drafter_create(const lng_drafter_numbers*, const lng_array*, int32_t, int32_t, lng_drafter** out) {
  if (out) *out = nullptr;
  return fail(LNG_ERR_UNSUPPORTED, "drafter not built yet");
}
extern "C" void lng_drafter_destroy(lng_drafter*) {}
extern "C" int lng_drafter_reset(lng_drafter*) { return LNG_ERR_UNSUPPORTED; }
extern "C" int64_t lng_drafter_length(const lng_drafter*) { return -1; }
extern "C" int lng_drafter_truncate(lng_drafter*, int64_t) { return LNG_ERR_UNSUPPORTED; }
extern "C" int lng_drafter_committed_codes(const lng_drafter*, uint8_t*) { return LNG_ERR_UNSUPPORTED; }
extern "C" int lng_drafter_commit(lng_drafter*, const int64_t*, int64_t, const int32_t*) { return LNG_ERR_UNSUPPORTED; }
extern "C" int lng_drafter_draft(lng_drafter*, int64_t, const int64_t*, int64_t, int32_t, int32_t, int64_t*, int64_t*,
                                 float*, uint8_t*) { return LNG_ERR_UNSUPPORTED; }
extern "C" int lng_drafter_trace(lng_drafter*, const int64_t*, int64_t, const int32_t*, int32_t, int64_t, uint8_t*,
                                 int64_t*, float*) { return LNG_ERR_UNSUPPORTED; }
extern "C" int lng_drafter_draft_batch(lng_drafter*, const int64_t*, int64_t, int64_t, int64_t, int64_t*, lng_stream_t) {
  return LNG_ERR_UNSUPPORTED;
}
