// TEST INFRASTRUCTURE ONLY. A stand-in for the Foundation part of Apple's
// metal-cpp, just large enough for the reference's host code (gym.h,
// model/ppo.h) to compile and run on the CPU: objects are plain heap objects
// and release() deletes them. Used by oracle/ref_host.cpp to run the
// reference's own host-side methods (parameter init, act, actGreedy,
// setLogStd, lastStats) on buffers this process fills.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

namespace NS {

using UInteger = std::size_t;
enum StringEncoding { UTF8StringEncoding = 4 };

class Object {
   public:
    virtual ~Object() = default;
    void release() { delete this; }
};

class String : public Object {
   public:
    static String* string(const char* s, StringEncoding) {
        String* o = new String;
        o->text = s ? s : "";
        return o;
    }
    const char* utf8String() const { return text.c_str(); }
    std::string text;
};

class Error : public Object {
   public:
    String* localizedDescription() const {
        static String none;
        none.text = "host stand-in";
        return &none;
    }
};

class AutoreleasePool : public Object {
   public:
    static AutoreleasePool* alloc() { return new AutoreleasePool; }
    AutoreleasePool* init() { return this; }
};

struct Range {
    UInteger location, length;
    static Range Make(UInteger loc, UInteger len) { return Range{loc, len}; }
};

}  // namespace NS
