// cxxopts.hpp -- a small command-line parser with the subset of the cxxopts
// API that the GLM drivers use (the reference's third-party/cxxopts submodule
// is empty in its checkout, so this is written from scratch):
//
//   cxxopts::Options opts("prog", "description");
//   opts.add_options()
//       ("nfeatures,X", "Number of features", cxxopts::value<long>()->default_value("25"))
//       ("h,help", "Print usage");
//   cxxopts::ParseResult r = opts.parse(argc, argv);
//   long nf = r["nfeatures"].as<long>();
//   if (r.count("help")) std::cout << opts.help();
//
// Accepted syntax: --name value, --name=value, -X value, -Xvalue, and bare
// --flag / -f for boolean options and options declared without a value.
// Errors throw cxxopts::exceptions::exception (unknown option, missing or
// unparsable value, option given twice).
#pragma once

#include <cctype>
#include <cerrno>
#include <cstdlib>
#include <limits>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

namespace cxxopts {

namespace exceptions {
class exception : public std::runtime_error {
   public:
    explicit exception(const std::string& what) : std::runtime_error(what) {}
};
class no_such_option : public exception {
   public:
    explicit no_such_option(const std::string& name) : exception("Option '" + name + "' does not exist") {}
};
class missing_argument : public exception {
   public:
    explicit missing_argument(const std::string& name) : exception("Option '" + name + "' is missing an argument") {}
};
class incorrect_argument_type : public exception {
   public:
    explicit incorrect_argument_type(const std::string& text)
        : exception("Argument '" + text + "' failed to parse") {}
};
class option_already_exists : public exception {
   public:
    explicit option_already_exists(const std::string& name) : exception("Option '" + name + "' already exists") {}
};
class option_has_no_value : public exception {
   public:
    explicit option_has_no_value(const std::string& name) : exception("Option '" + name + "' has no value") {}
};
}  // namespace exceptions

namespace detail {

template <typename T>
T parse_text(const std::string& text) {
    if constexpr (std::is_same_v<T, std::string>) {
        return text;
    } else if constexpr (std::is_same_v<T, bool>) {
        if (text == "true" || text == "1" || text == "yes" || text == "on") return true;
        if (text == "false" || text == "0" || text == "no" || text == "off") return false;
        throw exceptions::incorrect_argument_type(text);
    } else if constexpr (std::is_integral_v<T>) {
        if (text.empty()) throw exceptions::incorrect_argument_type(text);
        errno = 0;
        char* end = nullptr;
        if constexpr (std::is_signed_v<T>) {
            const long long v = std::strtoll(text.c_str(), &end, 0);
            if (errno != 0 || *end != '\0' || v < static_cast<long long>(std::numeric_limits<T>::min()) ||
                v > static_cast<long long>(std::numeric_limits<T>::max()))
                throw exceptions::incorrect_argument_type(text);
            return static_cast<T>(v);
        } else {
            if (text[0] == '-') throw exceptions::incorrect_argument_type(text);
            const unsigned long long v = std::strtoull(text.c_str(), &end, 0);
            if (errno != 0 || *end != '\0' || v > static_cast<unsigned long long>(std::numeric_limits<T>::max()))
                throw exceptions::incorrect_argument_type(text);
            return static_cast<T>(v);
        }
    } else if constexpr (std::is_floating_point_v<T>) {
        if (text.empty()) throw exceptions::incorrect_argument_type(text);
        errno = 0;
        char* end = nullptr;
        const long double v = std::strtold(text.c_str(), &end);
        if (errno != 0 || *end != '\0') throw exceptions::incorrect_argument_type(text);
        return static_cast<T>(v);
    } else {
        static_assert(!sizeof(T), "unsupported option type");
    }
}

}  // namespace detail

// Type-erased description of an option's value.
class Value : public std::enable_shared_from_this<Value> {
   public:
    virtual ~Value() = default;
    virtual bool is_boolean() const = 0;
    virtual void check(const std::string& text) const = 0;  // throws if unparsable
    std::shared_ptr<Value> default_value(const std::string& text) {
        check(text);
        default_ = text;
        has_default_ = true;
        return shared_from_this();
    }
    std::shared_ptr<Value> implicit_value(const std::string& text) {
        check(text);
        implicit_ = text;
        has_implicit_ = true;
        return shared_from_this();
    }
    bool has_default() const { return has_default_; }
    const std::string& get_default() const { return default_; }
    bool has_implicit() const { return has_implicit_ || is_boolean(); }
    std::string get_implicit() const { return has_implicit_ ? implicit_ : std::string("true"); }

   private:
    std::string default_, implicit_;
    bool has_default_ = false, has_implicit_ = false;
};

template <typename T>
class TypedValue : public Value {
   public:
    bool is_boolean() const override { return std::is_same_v<T, bool>; }
    void check(const std::string& text) const override { (void)detail::parse_text<T>(text); }
};

template <typename T>
std::shared_ptr<Value> value() {
    return std::make_shared<TypedValue<T>>();
}

// One parsed option: its text (given or default) and how often it was given.
class OptionValue {
   public:
    OptionValue() = default;
    OptionValue(std::string name, std::string text, bool has_value, size_t count)
        : name_(std::move(name)), text_(std::move(text)), has_value_(has_value), count_(count) {}
    template <typename T>
    T as() const {
        if (!has_value_) throw exceptions::option_has_no_value(name_);
        return detail::parse_text<T>(text_);
    }
    size_t count() const { return count_; }

   private:
    std::string name_, text_;
    bool has_value_ = false;
    size_t count_ = 0;
};

class ParseResult {
   public:
    ParseResult() = default;
    explicit ParseResult(std::map<std::string, OptionValue> values, std::vector<std::string> unmatched)
        : values_(std::move(values)), unmatched_(std::move(unmatched)) {}
    const OptionValue& operator[](const std::string& name) const {
        const auto it = values_.find(name);
        if (it == values_.end()) throw exceptions::no_such_option(name);
        return it->second;
    }
    size_t count(const std::string& name) const {
        const auto it = values_.find(name);
        return it == values_.end() ? 0 : it->second.count();
    }
    const std::vector<std::string>& unmatched() const { return unmatched_; }

   private:
    std::map<std::string, OptionValue> values_;
    std::vector<std::string> unmatched_;
};

class Options {
    struct Spec {
        std::string long_name, short_name, description;
        std::shared_ptr<Value> value;  // null: plain flag
    };

   public:
    class Adder {
       public:
        explicit Adder(Options& o) : o_(o) {}
        Adder& operator()(const std::string& names, const std::string& description,
                          std::shared_ptr<Value> value = nullptr) {
            o_.add(names, description, std::move(value));
            return *this;
        }

       private:
        Options& o_;
    };

    Options(std::string program, std::string description = "")
        : program_(std::move(program)), description_(std::move(description)) {}

    Adder add_options(const std::string& /*group*/ = "") { return Adder(*this); }

    ParseResult parse(int argc, const char* const* argv) const {
        std::map<std::string, std::string> given;  // long name -> text
        std::map<std::string, size_t> counts;
        std::vector<std::string> unmatched;
        for (int i = 1; i < argc; ++i) {
            const std::string arg = argv[i];
            if (arg.size() >= 2 && arg[0] == '-' && !(arg.size() > 1 && (std::isdigit(arg[1]) || arg[1] == '.'))) {
                std::string name, text;
                bool inline_text = false;
                const Spec* s = nullptr;
                if (arg[1] == '-') {
                    const auto eq = arg.find('=');
                    name = arg.substr(2, eq == std::string::npos ? std::string::npos : eq - 2);
                    if (eq != std::string::npos) {
                        text = arg.substr(eq + 1);
                        inline_text = true;
                    }
                    s = find_long(name);
                } else {
                    name = arg.substr(1, 1);
                    if (arg.size() > 2) {
                        text = arg.substr(arg[2] == '=' ? 3 : 2);
                        inline_text = true;
                    }
                    s = find_short(name);
                }
                if (s == nullptr) throw exceptions::no_such_option(name);
                if (!s->value) {
                    if (inline_text) throw exceptions::incorrect_argument_type(arg);
                    given[s->long_name] = "true";
                } else if (inline_text) {
                    s->value->check(text);
                    given[s->long_name] = text;
                } else if (s->value->is_boolean()) {
                    given[s->long_name] = s->value->get_implicit();
                } else {
                    if (i + 1 >= argc) throw exceptions::missing_argument(s->long_name);
                    text = argv[++i];
                    s->value->check(text);
                    given[s->long_name] = text;
                }
                ++counts[s->long_name];
            } else {
                unmatched.push_back(arg);
            }
        }
        std::map<std::string, OptionValue> values;
        for (const Spec& s : specs_) {
            const auto g = given.find(s.long_name);
            const size_t n = counts.count(s.long_name) ? counts.at(s.long_name) : 0;
            OptionValue v;
            if (g != given.end()) {
                v = OptionValue(s.long_name, g->second, true, n);
            } else if (s.value && s.value->has_default()) {
                v = OptionValue(s.long_name, s.value->get_default(), true, 0);
            } else if (!s.value) {
                v = OptionValue(s.long_name, "false", true, 0);
            } else {
                v = OptionValue(s.long_name, "", false, 0);
            }
            values[s.long_name] = v;
            if (!s.short_name.empty()) values[s.short_name] = v;
        }
        return ParseResult(std::move(values), std::move(unmatched));
    }

    std::string help() const {
        std::ostringstream os;
        os << description_ << "\nUsage:\n  " << program_ << " [OPTION...]\n\n";
        for (const Spec& s : specs_) {
            std::string left = "  ";
            left += s.short_name.empty() ? "    " : ("-" + s.short_name + ", ");
            left += "--" + s.long_name;
            if (s.value && !s.value->is_boolean()) left += " arg";
            if (left.size() < 34) left.resize(34, ' ');
            os << left << " " << s.description;
            if (s.value && s.value->has_default() && !s.value->is_boolean())
                os << " (default: " << s.value->get_default() << ")";
            os << "\n";
        }
        return os.str();
    }

   private:
    void add(const std::string& names, const std::string& description, std::shared_ptr<Value> value) {
        Spec s;
        const auto comma = names.find(',');
        std::string a = names.substr(0, comma), b = comma == std::string::npos ? "" : names.substr(comma + 1);
        auto trim = [](std::string x) {
            while (!x.empty() && x.front() == ' ') x.erase(x.begin());
            while (!x.empty() && x.back() == ' ') x.pop_back();
            return x;
        };
        a = trim(a);
        b = trim(b);
        if (b.empty()) {
            s.long_name = a;
        } else if (a.size() == 1) {
            s.short_name = a;
            s.long_name = b;
        } else {
            s.long_name = a;
            s.short_name = b;
        }
        if (s.long_name.empty() || s.short_name.size() > 1) throw exceptions::exception("bad option names: " + names);
        if (find_long(s.long_name) || (!s.short_name.empty() && find_short(s.short_name)))
            throw exceptions::option_already_exists(names);
        s.description = description;
        s.value = std::move(value);
        specs_.push_back(std::move(s));
    }
    const Spec* find_long(const std::string& n) const {
        for (const Spec& s : specs_)
            if (s.long_name == n) return &s;
        return nullptr;
    }
    const Spec* find_short(const std::string& n) const {
        for (const Spec& s : specs_)
            if (s.short_name == n) return &s;
        return nullptr;
    }

    std::string program_, description_;
    std::vector<Spec> specs_;
};

}  // namespace cxxopts
